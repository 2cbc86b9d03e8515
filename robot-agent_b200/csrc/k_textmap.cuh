// The text model inside the keyframe chain (ObjectMap with setTextModel / setClassKinds).
//
//  - k_obs_text: apObsStructural's label part (scenemap src/objmap.cpp:547-564): the
//    observation's apLabelLogLik (kept per detection: apAddView adds the same values to the
//    object later), the probability mass of structure labels (ps) and of structural-object labels
//    (pso), the most likely structural-object shape group (door / window, stairs, pillar: the
//    size rules' sh) and the single-fragment top label (top_p, top_lab: the name veto).
//  - k_rename: apRename (objmap.cpp:1227-1240) -> apName (objprob.cpp:396-455) of every object
//    whose rename is due, one warp per object: after the merge pass (merged objects,
//    objmap.cpp:1217), after the update (objects seen in the keyframe, :1008) and after whole-view
//    answers (:1365).  The posterior, name, top label, entropy and the class (cls = name) are
//    written back; gp_so caches apGroupProb over the structure and structural-object labels,
//    which the association and merge guards read.
// Device exp / log / log1p may differ from the host libm in the last bit, so label
// log-likelihoods and posteriors match the reference to ~1e-7 relative.
#pragma once
#include "k_assoc.cuh"
#include "k_text.cuh"

#define OBT_THREADS 256
#define RN_WARPS 4

__global__ void __launch_bounds__(OBT_THREADS) k_obs_text(Batch B) {
  extern __shared__ __align__(16) unsigned char ot_raw[];
  const int m = B.map0 + blockIdx.y, k = blockIdx.x, tid = threadIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active || k >= F.n_det || !F.emb || B.txt.dim != B.D) return;
  ObsRec* O = &B.obs[(size_t)m * B.max_det + k];
  const TextDev& T = B.txt;
  const int C = T.n_labels;
  float* zs = (float*)ot_raw;
  float* best = zs + T.dim;
  float* ll = B.llz + ((size_t)m * B.max_det + k) * C;
  for (int i = tid; i < T.dim; i += blockDim.x)
    zs[i] = F.emb_dtype == SMG_EMB_BF16 ? __uint_as_float((uint32_t)((const uint16_t*)F.emb)[(size_t)k * B.D + i] << 16)
                                        : ((const float*)F.emb)[(size_t)k * B.D + i];
  __syncthreads();
  label_loglik_block(T, zs, best, ll);
  if (tid != 0) return;
  // sums in label order, as the reference adds them (objmap.cpp:551-563)
  double q = 0, qo = 0, qsh[4] = {0, 0, 0, 0}, top_p = 0;
  int top_lab = -1;
  for (int l = 0; l < C; ++l) {
    if (ll[l] <= -1e29f) continue;
    const float e = expf(ll[l]);
    const int kd = kind_of(B, l);
    if (kd == KIND_STRUCTURE) q += (double)e;
    if (kd == KIND_STRUCT_OBJ) {
      qo += (double)e;
      qsh[T.so_shape ? T.so_shape[l] & 3 : 0] += (double)e;
    }
    if ((double)e > top_p) { top_p = (double)e; top_lab = l; }
  }
  int sh = 1;   // std::max_element(qsh + 1, qsh + 4): the first largest
  for (int i = 2; i < 4; ++i)
    if (qsh[i] > qsh[sh]) sh = i;
  O->ps = q;
  O->pso = qo;
  O->top_p = top_p;
  O->top_lab = top_lab;
  O->so_sh = sh;
}

// apRename -> apName of object o (global record index og) by one warp; lp, up: the warp's
// 2 x C doubles of shared scratch.
DEV void ap_rename_warp(const Batch& B, ObjRec& o, size_t og, double* lp, double* up) {
  const TextDev& T = B.txt;
  const smg_params& P = B.p;
  const int C = T.n_labels, lane = threadIdx.x & 31;
  const float* Lf = B.lfrag + og * C;
  const float* Lw = B.lwhole + og * C;
  float* post = B.post + og * C;
  const double size = smax(smax(o.hi[0] - o.lo[0], o.hi[1] - o.lo[1]), o.hi[2] - o.lo[2]);
  double lw = 0;
  if (o.has_lfrag) lw += o.lw_frag;
  if (o.has_lwhole) lw += P.whole_w * o.lw_whole;
  if (!(lw > 0)) return;   // no image evidence yet: the name stays as it is
  const bool geo3 = o.geo == 3;   // L_geo (apRename): thin plane on a wall line
  const double lam = lw > P.name_wmax ? P.name_wmax / lw : 1.0;   // name_lambda
  const double ls = log(smax(size, 0.02));
  for (int c = lane; c < C; c += 32) {
    float L = 0.f;
    if (o.has_lfrag) L += Lf[c];
    if (o.has_lwhole) L += (float)(P.whole_w * (double)Lw[c]);
    double v = lam * (double)L;
    if (L < -1e29f || (double)L <= -60.0 * lw) v = -1e300;
    if (T.log_prior) v += (double)T.log_prior[c];
    if (geo3 && (kind_of(B, c) == KIND_STRUCT_OBJ || (T.flat_ok && T.flat_ok[c]))) v += (double)(float)P.geo_w;
    if (T.ls_sd && T.ls_sd[c] > 0) {
      const double zz = (ls - (double)T.ls_mu[c]) / (double)T.ls_sd[c];
      v += P.size_w * (-0.5 * zz * zz - log((double)T.ls_sd[c]));
    }
    lp[c] = v;
  }
  __syncwarp();
  if (lane == 0) {
    // softmax_post (objprob_math.h:102-120), dead = -1e299, no rest group
    const double dead = -1e299;
    double mx = dead;
    bool any = false;
    for (int c = 0; c < C; ++c)
      if (lp[c] > dead) { mx = any ? smax(mx, lp[c]) : lp[c]; any = true; }
    double se = 0;
    for (int c = 0; c < C; ++c)
      if (lp[c] > dead) se += exp(lp[c] - mx);
    double H = 0;
    int best = -1;
    for (int c = 0; c < C; ++c) {
      if (!(lp[c] > dead)) { post[c] = 0.f; continue; }
      const double q = exp(lp[c] - mx) / se;
      if (q > 1e-12) H -= q * log(q);
      post[c] = (float)q;
      if (best < 0 || q > (double)post[best]) best = c;
    }
    const float top_p = best >= 0 ? post[best] : 0.f;
    int name_lab, rolled = 0;
    float name_p;
    if (best >= 0 && (double)top_p >= P.name_tau) {
      name_lab = best;
      name_p = top_p;
    } else {   // hypernym roll-up: probability under each ancestor (8 levels), the deepest one >= name_tau
      for (int c = 0; c < C; ++c) up[c] = 0.0;
      for (int c = 0; c < C; ++c) {
        int p = T.parent ? T.parent[c] : -1;
        for (int g = 0; p >= 0 && p < C && g < 8; ++g, p = T.parent[p]) up[p] += (double)post[c];
      }
      int gsel = -1, gdep = 0;
      for (int c = 0; c < C; ++c) {
        int p = T.parent ? T.parent[c] : -1, dpt = 0;
        while (p >= 0 && p < C && dpt < 8) { ++dpt; p = T.parent[p]; }
        const double ug = gsel >= 0 ? up[gsel] : 0.0;
        if (up[c] >= P.name_tau && (gsel < 0 || dpt > gdep || (dpt == gdep && up[c] > ug))) { gsel = c; gdep = dpt; }   // better_hyper
      }
      rolled = 1;
      if (gsel >= 0) { name_lab = gsel; name_p = (float)up[gsel]; }
      else if (T.object_label >= 0) { name_lab = T.object_label; name_p = top_p; }
      else { name_lab = best; name_p = top_p; rolled = 0; }
    }
    o.name_H = (float)H;
    o.top_lab = best;
    o.top_p = top_p;
    o.rolled = rolled;
    o.name_lab = name_lab;
    o.name_p = name_p;
    o.has_post = 1;
    ++o.post_ver;
    if (name_lab >= 0) o.cls = name_lab;   // apRename (objmap.cpp:1239)
    double g = 0;   // apGroupProb over the structure and structural-object labels, label order
    for (int c = 0; c < C; ++c) {
      const int kd = kind_of(B, c);
      if (kd == KIND_STRUCTURE || kd == KIND_STRUCT_OBJ) g += (double)post[c];
    }
    o.gp_so = g;
  }
  __syncwarp();
}

// Renames that are due, list order, one warp per object.
__global__ void __launch_bounds__(RN_WARPS * 32) k_rename(Batch B) {
  extern __shared__ __align__(16) unsigned char rn_raw[];
  const int m = B.map0 + blockIdx.y, wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (!B.frames[m].active || !B.text_on) return;
  const int C = B.txt.n_labels;
  double* lp = (double*)rn_raw + (size_t)wid * 2 * C;
  double* up = lp + C;
  const int n = B.maps[m].n_obj;
  for (int i = blockIdx.x * RN_WARPS + wid; i < n; i += gridDim.x * RN_WARPS) {
    const int s = slot_at(B, m, i);
    if (!INB(s, B.O, 910)) continue;
    ObjRec& o = B.objs[oglob(B, m, s)];
    if (!o.rename) continue;
    ap_rename_warp(B, o, oglob(B, m, s), lp, up);
    if (lane == 0) o.rename = 0;
    __syncwarp();
  }
}
