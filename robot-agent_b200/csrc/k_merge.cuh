// Object-object merge pass at the start of a keyframe (apMergePass, scenemap src/objmap.cpp:
// 1154-1225, apPairObj :1118-1135, da::absorbObject da/src/merge.cpp:32-82, apMerge
// objprob.cpp:358-394).
//
// k_merge_gate tests every pair i < j (box-gap and size gates) and lists the survivors;
// k_merge_pairs then evaluates them, a warp per pair taken from the map's list: the contact
// fraction of a <= 2*contact_samples sample of the smaller cloud against the larger cloud's
// contact set, and the symmetric embedding cosine (each object's mean direction against the
// other's vectors).  Pairs with P >= merge_p go to a
// per-map candidate list.  (The reference's pair cache only skips recomputing identical inputs,
// so evaluating every gated pair gives the same P.)
// k_merge_apply: one CTA per map sorts the candidates by P and merges greedily, each object at
// most once per pass, as the reference does.
#pragma once
#include "k_life.cuh"

#define MP_CTAS 8
#define MGL_CAP 65536   // gated pairs per map and frame
#define MP_SMEM(O) ((size_t)(O) * (7 * 8 + 8))   // k_merge_gate: boxes, guard mass, states, guard flags

// p-th pair (i < j) of n objects in row-major order of the upper triangle
DEV void pair_of(long long p, int n, int* pi, int* pj) {
  auto rowstart = [&](long long i) { return i * (2LL * n - i - 1) / 2; };
  long long i = (long long)((2.0 * n - 1 - sqrt((2.0 * n - 1) * (2.0 * n - 1) - 8.0 * (double)p)) / 2.0);
  if (i < 0) i = 0;
  while (i > 0 && rowstart(i) > p) --i;
  while (i + 1 < n && rowstart(i + 1) <= p) ++i;
  *pi = (int)i;
  *pj = (int)(p - rowstart(i) + i + 1);
}

// Pair gating: the 8 CTAs of a map share the pairs and append the gated ones to the map's list.
__global__ void __launch_bounds__(256) k_merge_gate(Batch B) {
  extern __shared__ unsigned char smem_raw[];
  const int m = B.map0 + blockIdx.y, tid = threadIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active) return;
  const MapRec& R = B.maps[m];
  const smg_params& P = B.p;
  const int n = R.n_obj;
  if (n < 2) return;
  double* slo = (double*)smem_raw;
  double* shi = slo + 3 * (size_t)B.O;
  double* sgp = shi + 3 * (size_t)B.O;       // structure-group posterior mass
  int* sst = (int*)(sgp + (size_t)B.O);
  int* sfl = sst + B.O;                      // bit 0: post, bit 1: struct-looking, bit 2: flat name
  // 1. stage the gate inputs of every object (parallel loads)
  for (int b = tid; b < n; b += blockDim.x) {
    const ObjRec& o = obj_at(B, m, b);
    for (int k = 0; k < 3; ++k) { slo[3 * b + k] = o.lo[k]; shi[3 * b + k] = o.hi[k]; }
    sst[b] = o.held_by >= 0 ? 1 : o.state;   // held objects are left out like gone ones (objmap.cpp:1162-1165)
    sgp[b] = o.gp_so;
    sfl[b] = (o.has_post ? 1 : 0) | (2 * o.n_struct_look > o.n_ap_obs ? 2 : 0) | (flat_named(B, o) ? 4 : 0);
  }
  __syncthreads();
  // 2. box-gap and size gates of all pairs (objmap.cpp:1160-1173); this CTA takes every
  //    MP_CTAS-th pair
  const double gate2 = P.gate * P.gate;
  const long long npair = (long long)n * (n - 1) / 2;
  for (long long p = (long long)blockIdx.x * blockDim.x + tid; p < npair; p += (long long)gridDim.x * blockDim.x) {
    int i, j;
    pair_of(p, n, &i, &j);
    if (sst[i] == 1 || sst[j] == 1) continue;
    double g2 = 0;
    bool too_big = false;
    for (int k = 0; k < 3; ++k) {
      const double g = smax3(0.0, slo[3 * i + k] - shi[3 * j + k], slo[3 * j + k] - shi[3 * i + k]);
      g2 += g * g;
      too_big = too_big || smax(shi[3 * i + k], shi[3 * j + k]) - smin(slo[3 * i + k], slo[3 * j + k]) > P.max_ext;
    }
    if (g2 > gate2 || too_big) continue;
    if ((sfl[i] & 1) && (sfl[j] & 1)) {   // structure guards (objmap.cpp:1174-1181)
      const double sa = sgp[i], sb = sgp[j];
      if ((sa >= P.guard_obj && sb <= P.guard_obs) || (sb >= P.guard_obj && sa <= P.guard_obs)) continue;
      if (P.struct_look_block) {
        const bool la = sfl[i] & 2, lb = sfl[j] & 2;
        if ((la && !lb && sb < 0.5) || (lb && !la && sa < 0.5)) continue;
      }
    }
    if (((sfl[i] | sfl[j]) & 4) &&   // a flat wall-mounted name past its size (objmap.cpp:1182-1184)
        smax(smax(shi[3 * i], shi[3 * j]) - smin(slo[3 * i], slo[3 * j]), smax(shi[3 * i + 1], shi[3 * j + 1]) - smin(slo[3 * i + 1], slo[3 * j + 1])) >
            P.flat_max_w)
      continue;
    const int q = atomicAdd(&B.mgl_n[m], 1);
    if (q < MGL_CAP) B.mgl[(size_t)m * MGL_CAP + q] = i << 16 | j;
    else set_err(&B.maps[m], SMG_E_ARGS);
  }
}

// Pair evaluation: every warp of the map's CTAs takes the next gated pair of the map's list, so
// a slow pair (cosines against all views, contact test) holds one warp, not a CTA's share.
__global__ void __launch_bounds__(256) k_merge_pairs(Batch B) {
  const int m = B.map0 + blockIdx.y, lane = threadIdx.x & 31;
  const FrameDev& F = B.frames[m];
  if (!F.active) return;
  const MapRec& R = B.maps[m];
  const smg_params& P = B.p;
  if (R.n_obj < 2) return;
  const int ng = min(B.mgl_n[m], MGL_CAP);
  for (;;) {
    int g = 0;
    if (lane == 0) g = atomicAdd(&B.mgl_n[B.M + m], 1);
    g = __shfl_sync(0xffffffffu, g, 0);
    if (g >= ng) break;
    const int key = B.mgl[(size_t)m * MGL_CAP + g];
    const int i = key >> 16, j = key & 0xffff;
    const int si = slot_at(B, m, i), sj = slot_at(B, m, j);
    const size_t ogi = oglob(B, m, si), ogj = oglob(B, m, sj);
    const ObjRec& a = B.objs[ogi];
    const ObjRec& b = B.objs[ogj];
    const int scn_i = B.clouds[cglob(B, m, a.cloud_slot)].n, scn_j = B.clouds[cglob(B, m, b.cloud_slot)].n;
    const bool a_small = scn_i <= scn_j;
    const ObjRec& sm = a_small ? a : b;
    const ObjRec& lg = a_small ? b : a;
    const size_t css = cglob(B, m, sm.cloud_slot), csl = cglob(B, m, lg.cloud_slot);
    const int cn = a_small ? scn_i : scn_j;
    const int stp = max(1, cn / max(1, P.contact_samples));
    const int nsp = cn > 0 ? (cn + stp - 1) / stp : 0;
    // cached cosine and contact of an unchanged pair
    const uint32_t ca = B.clouds[cglob(B, m, a.cloud_slot)].version, cb = B.clouds[cglob(B, m, b.cloud_slot)].version;
    PairCacheRec& pc = B.pcache[(size_t)m * PCACHE_SLOTS + (hmix(((uint64_t)a.id << 32) | b.id) & (PCACHE_SLOTS - 1))];
    const bool hit = pc.ida == a.id && pc.idb == b.id && pc.va == a.ver && pc.vb == b.ver && pc.ca == ca && pc.cb == cb;
    double cs = -2, contact = 0.0;
    if (hit) {
      cs = pc.cs;
      contact = pc.contact;
    } else {
      if (a.nrm_frag > 0) cs = smax(cs, cos_max_warp(B, ogj, b, B.mu + ogi * B.D));
      if (b.nrm_frag > 0) cs = smax(cs, cos_max_warp(B, ogi, a, B.mu + ogj * B.D));
      const int hits = contact_hits_cloud_warp(B, csl, css, stp, nsp, P.contact_cell);
      contact = (nsp > 0 && B.clouds[csl].cn > 0) ? (double)hits / (double)nsp : 0.0;
      __syncwarp();
      if (lane == 0) {
        pc.ida = a.id; pc.idb = b.id; pc.va = a.ver; pc.vb = b.ver; pc.ca = ca; pc.cb = cb;
        pc.cs = cs;
        pc.contact = contact;
      }
    }
    // name-distribution overlap (objmap.cpp:1129-1133): Bhattacharyya coefficient - 0.5, label order
    double f6 = 0;
    const bool names = a.has_post && b.has_post;
    if (names && lane == 0) {
      const int C = B.txt.n_labels;
      const float* pa = B.post + ogi * C;
      const float* pb2 = B.post + ogj * C;
      double bc = 0;
      for (int l = 0; l < C; ++l) bc += sqrt((double)pa[l] * pb2[l]);
      f6 = bc - 0.5;
    }
    if (lane == 0) {
      const double p = pair_p(sm.lo, sm.hi, sm.pos, contact, lg.lo, lg.hi, lg.pos, cs, P, true, nullptr, f6);
      if (p >= P.merge_p) {
        const int c = atomicAdd(&B.mcand_n[m], 1);
        if (c < B.O * 8) {
          B.mcand_p[(size_t)m * B.O * 8 + c] = p;
          B.mcand_ab[((size_t)m * B.O * 8 + c) * 2] = a.id;
          B.mcand_ab[((size_t)m * B.O * 8 + c) * 2 + 1] = b.id;
          B.mcand_key[(size_t)m * B.O * 8 + c] = (uint32_t)i << 16 | (uint32_t)j;
        } else {
          set_err(&B.maps[m], SMG_E_ARGS);
        }
      }
    }
    __syncwarp();
  }
}

__global__ void __launch_bounds__(512) k_merge_apply(Batch B) {
  __shared__ BlockScratch bs;
  __shared__ int hist[SEL_HIST(1)];
  __shared__ int sh_go, sh_ka, sh_kb, sh_pkb, nused, sh_pa, sh_pb;
  __shared__ uint32_t used[2 * 256];
  const int m = B.map0 + blockIdx.x, tid = threadIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active) return;
  MapRec* R = &B.maps[m];
  const smg_params& P = B.p;
  const double t = F.stamp;
  const int nc = min(B.mcand_n[m], B.O * 8);
  double* cp = B.mcand_p + (size_t)m * B.O * 8;
  uint32_t* cab = B.mcand_ab + (size_t)m * B.O * 8 * 2;
  uint32_t* ckey = B.mcand_key + (size_t)m * B.O * 8;
  if (tid == 0) {
    R->n_evn = 0;
    nused = 0;
    // descending P; equal P keep the reference's enumeration order (pairs i < j in list order),
    // which is what its std::sort leaves for lists of up to 16 candidates (insertion sort)
    for (int i = 1; i < nc; ++i) {
      const double p = cp[i];
      const uint32_t x = cab[2 * i], y = cab[2 * i + 1], kk = ckey[i];
      int j = i;
      while (j > 0 && (cp[j - 1] < p || (cp[j - 1] == p && ckey[j - 1] > kk))) {
        cp[j] = cp[j - 1]; cab[2 * j] = cab[2 * j - 2]; cab[2 * j + 1] = cab[2 * j - 1]; ckey[j] = ckey[j - 1];
        --j;
      }
      cp[j] = p; cab[2 * j] = x; cab[2 * j + 1] = y; ckey[j] = kk;
    }
  }
  __syncthreads();
  const Work W = work_at(B, m, 0);
  float* xyz = B.cxyz + (size_t)m * B.max_det * 3 * B.pmax;
  uint8_t* rgb = (uint8_t*)(B.cpx + (size_t)m * B.max_det * 2 * B.pmax);
  for (int c = 0; c < nc; ++c) {
    // list positions of the pair's objects (findPos), searched by the whole block
    const uint32_t ia = cab[2 * c], ib = cab[2 * c + 1];
    if (tid == 0) { sh_pa = 0x7fffffff; sh_pb = 0x7fffffff; }
    __syncthreads();
    for (int i = tid; i < R->n_obj; i += blockDim.x) {
      const uint32_t id = obj_at(B, m, i).id;
      if (id == ia) atomicMin(&sh_pa, i);
      if (id == ib) atomicMin(&sh_pb, i);
    }
    __syncthreads();
    if (tid == 0) {
      sh_go = 0;
      bool u = false;
      for (int q = 0; q < nused; ++q) u = u || used[q] == ia || used[q] == ib;
      const int pa = sh_pa == 0x7fffffff ? -1 : sh_pa, pb = sh_pb == 0x7fffffff ? -1 : sh_pb;
      if (!u && pa >= 0 && pb >= 0 && nused + 2 <= 2 * 256) {
        int ka = pa, kb = pb;
        const ObjRec& A = obj_at(B, m, pa);
        const ObjRec& Bo = obj_at(B, m, pb);
        if (Bo.n_obs > A.n_obs || (Bo.n_obs == A.n_obs && ib < ia)) { ka = pb; kb = pa; }
        used[nused++] = ia;
        used[nused++] = ib;
        sh_ka = slot_at(B, m, ka);
        sh_kb = slot_at(B, m, kb);
        sh_pkb = kb;
        sh_go = 1;
        // da::absorb scalar part (merge.cpp:33-62)
        ObjRec& a = B.objs[oglob(B, m, sh_ka)];
        const ObjRec& b = B.objs[oglob(B, m, sh_kb)];
        const bool big = kind_of(B, a.cls) == KIND_STATIC ||   // bigPair (merge.cpp:25-29)
                         smax(smax(a.hi[0] - a.lo[0], a.hi[1] - a.lo[1]), smax(b.hi[0] - b.lo[0], b.hi[1] - b.lo[1])) > P.big;
        const double wa = smax((double)a.n_obs, 1.0), wb = smax((double)b.n_obs, 1.0);
        for (int k = 0; k < 3; ++k) {
          if (big) {
            a.lo[k] = smin(a.lo[k], b.lo[k]);
            a.hi[k] = smax(a.hi[k], b.hi[k]);
            a.pos[k] = 0.5 * (a.lo[k] + a.hi[k]);
            a.ext[k] = a.hi[k] - a.lo[k];
          } else {
            a.pos[k] = (a.pos[k] * wa + b.pos[k] * wb) / (wa + wb);
            a.ext[k] = (a.ext[k] * wa + b.ext[k] * wb) / (wa + wb);
            a.lo[k] = (a.lo[k] * wa + b.lo[k] * wb) / (wa + wb);
            a.hi[k] = (a.hi[k] * wa + b.hi[k] * wb) / (wa + wb);
          }
        }
        if (b.first_seen < a.first_seen) {
          a.first_seen = b.first_seen;
          for (int k = 0; k < 3; ++k) a.first_pos[k] = b.first_pos[k];
        }
        a.n_obs += b.n_obs;
        a.last_seen = smax(a.last_seen, b.last_seen);
        a.last_kf = smax(a.last_kf, b.last_kf);
        a.score = (a.score < b.score) ? b.score : a.score;
        a.max_det_z = smax(a.max_det_z, b.max_det_z);
        a.moved = a.moved || b.moved;
        a.misses = min(a.misses, b.misses);
        a.n_vis_miss += b.n_vis_miss;
        if (a.state != 0 && b.state == 0) a.state = 0;
        if (!a.parent) { a.parent = b.parent; for (int k = 0; k < 3; ++k) a.parent_rel[k] = b.parent_rel[k]; }
      }
    }
    __syncthreads();
    if (!sh_go) continue;
    const size_t oga = oglob(B, m, sh_ka), ogb = oglob(B, m, sh_kb);
    ObjRec& a = B.objs[oga];
    const ObjRec& b = B.objs[ogb];
    const size_t csa = cglob(B, m, a.cloud_slot), csb = cglob(B, m, b.cloud_slot);
    // cloud: b's points (org + p) into a (merge.cpp:64-75)
    const CloudRec& Cb = B.clouds[csb];
    const int nb = Cb.n;
    const float4* pb = B.cpts + csb * B.cap;
    const uint32_t* colb = B.crgb + csb * B.cap;
    if (!INB(3 * nb, 3 * B.max_det * B.pmax, 601)) continue;
    for (int i = tid; i < nb; i += blockDim.x) {
      const float4 p = pb[i];
      xyz[3 * i] = (float)(Cb.org[0] + (double)p.x);
      xyz[3 * i + 1] = (float)(Cb.org[1] + (double)p.y);
      xyz[3 * i + 2] = (float)(Cb.org[2] + (double)p.z);
      rgb[3 * i] = (uint8_t)(colb[i] & 255u);
      rgb[3 * i + 1] = (uint8_t)((colb[i] >> 8) & 255u);
      rgb[3 * i + 2] = (uint8_t)((colb[i] >> 16) & 255u);
    }
    __syncthreads();
    if (nb > 0) cloud_add(B, m, csa, xyz, rgb, nb, t, W, hist, bs);
    // apMerge: vectors (objprob.cpp:359-377): whole views were parts of the merged object, so
    // r_frag += a.r_whole, += b.r_frag, += b.r_whole (each added only when it holds a vector)
    float* ra = B.rfrag + oga * B.D;
    const float* rb = B.rfrag + ogb * B.D;
    const float* raw = B.rwhole + oga * B.D;
    const float* rbw = B.rwhole + ogb * B.D;
    const bool aw = a.has_whole != 0, bw = b.has_whole != 0;
    for (int i = tid; i < B.D; i += blockDim.x) {
      float x = ra[i];
      if (aw) x += raw[i];
      x += rb[i];
      if (bw) x += rbw[i];
      ra[i] = x;
    }
    if (B.text_on) {   // the label vectors in the same order (a vector is added only when it is not empty)
      const int C = B.txt.n_labels;
      float* La = B.lfrag + oga * C;
      const float* Law = B.lwhole + oga * C;
      const float* Lb = B.lfrag + ogb * C;
      const float* Lbw = B.lwhole + ogb * C;
      const bool hf = a.has_lfrag, hw = a.has_lwhole, bf = b.has_lfrag, bhw = b.has_lwhole;
      for (int l = tid; l < C; l += blockDim.x) {
        float x = hf ? La[l] : 0.f;
        if (hw) x += Law[l];
        if (bf) x += Lb[l];
        if (bhw) x += Lbw[l];
        La[l] = x;
      }
    }
    __syncthreads();
    if (tid == 0 && B.text_on) {
      a.has_lfrag = a.has_lfrag || a.has_lwhole || b.has_lfrag || b.has_lwhole;
      a.has_lwhole = 0;
    }
    // views: a's and b's in one list, fragments, stable by kappa desc, top-k (objprob.cpp:382-385)
    __shared__ int vsrc[2 * SMG_TOPK_MAX + 2], vphys[2 * SMG_TOPK_MAX + 2], dstp[2 * SMG_TOPK_MAX + 2], nkeep;
    __shared__ float vk[2 * SMG_TOPK_MAX + 2];
    __shared__ double vs[2 * SMG_TOPK_MAX + 2];
    if (tid == 0) {
      int nv = 0;
      for (int v = 0; v < a.n_views; ++v) { vsrc[nv] = 0; vphys[nv] = a.view_slot[v]; vk[nv] = a.vkappa[v]; vs[nv] = a.vstamp[v]; ++nv; }
      for (int v = 0; v < b.n_views; ++v) { vsrc[nv] = 1; vphys[nv] = b.view_slot[v]; vk[nv] = b.vkappa[v]; vs[nv] = b.vstamp[v]; ++nv; }
      for (int i = 1; i < nv; ++i) {
        const int s0 = vsrc[i], p0 = vphys[i];
        const float k0 = vk[i];
        const double t0 = vs[i];
        int j = i;
        while (j > 0 && vk[j - 1] < k0) { vsrc[j] = vsrc[j - 1]; vphys[j] = vphys[j - 1]; vk[j] = vk[j - 1]; vs[j] = vs[j - 1]; --j; }
        vsrc[j] = s0; vphys[j] = p0; vk[j] = k0; vs[j] = t0;
      }
      nkeep = min(nv, B.topk);
      int usedm = 0;
      for (int v = 0; v < nkeep; ++v) if (vsrc[v] == 0) usedm |= 1 << vphys[v];
      for (int v = 0; v < nkeep; ++v) {
        if (vsrc[v] == 0) { dstp[v] = vphys[v]; continue; }
        int f = 0;
        while (usedm & (1 << f)) ++f;
        usedm |= 1 << f;
        dstp[v] = f;
      }
    }
    __syncthreads();
    for (int v = 0; v < nkeep; ++v) {
      if (vsrc[v] != 1) continue;
      if (!INB(vphys[v], B.topk + 1, 602) || !INB(dstp[v], B.topk + 1, 603)) continue;
      const uint16_t* src = B.views + (ogb * (B.topk + 1) + vphys[v]) * B.D;
      uint16_t* dst = B.views + (oga * (B.topk + 1) + dstp[v]) * B.D;
      for (int i = tid; i < B.D; i += blockDim.x) dst[i] = src[i];
    }
    __syncthreads();
    if (tid == 0) {
      for (int v = 0; v < nkeep; ++v) { a.view_slot[v] = dstp[v]; a.vkappa[v] = vk[v]; a.vstamp[v] = vs[v]; a.vwhole[v] = 0; }
      a.n_views = nkeep;
      ++a.ver;
      a.k_frag += (a.k_whole + b.k_frag) + b.k_whole;
      a.k_whole = 0;
      a.has_whole = 0;
      a.nrm_whole = 0;
      a.n_whole = 0;
      a.whole_kappa = 0;
      a.need_whole = 1;
      // cams: append b's, keep the newest 32
      for (int q = 0; q < b.n_cams; ++q) cam_push(a, cam_at(b, q));
      for (int k = 0; k < 3; ++k) a.P[k] = merge_var(a.P[k], b.P[k]);
      a.n_wall_obs += b.n_wall_obs;
      a.n_ap_obs += b.n_ap_obs;
      a.n_struct_look += b.n_struct_look;
      a.wall_like = a.wall_like && b.wall_like;
      a.confirmed = a.confirmed || b.confirmed;
      // label evidence (objprob.cpp:370-374): L_frag += a.L_whole, b.L_frag, b.L_whole
      a.lw_frag += (a.lw_whole + b.lw_frag) + b.lw_whole;
      a.lw_whole = 0;
      a.rename = B.text_on;   // apRename after the absorb (objmap.cpp:1217)
      ++R->st.n_merge;
      const uint32_t did = b.id;
      { const int pe = sh_pkb; if (INB(pe, R->n_obj, 604)) erase_pos(B, m, pe, false); }   // b's position (findPos)
      for (int i = 0; i < R->n_obj; ++i) {   // remapId(did, kid) (objmap.cpp:1222) on the parent links
        ObjRec& o = B.objs[oglob(B, m, slot_at(B, m, i))];
        if (o.parent == did) o.parent = a.id;
      }
      push_event(B, m, t, a, 7, (1u << 24) | (uint32_t)R->n_evn++);
    }
    __syncthreads();
    refresh_nrm(B, oga, bs);
    if (B.clouds[csa].cver != B.clouds[csa].version) contact_rebuild(B, csa, bs);
  }
  // reset the per-frame association flags (list positions)
  for (int i = tid; i < B.O; i += blockDim.x) {
    B.touched[(size_t)m * B.O + i] = 0;
    B.obj_hit[(size_t)m * B.O + i] = 0;
  }
  if (tid == 0) B.mcand_n[m] = 0;
}
