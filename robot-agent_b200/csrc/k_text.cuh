// Text-model label posterior on the device: apLabelLogLik (scenemap src/objprob.cpp:287-310)
// and apName (objprob.cpp:396-455, with objprob_math.h label_weight/name_lambda/softmax_post/
// better_hyper).
//
// k_label_loglik: one CTA per embedding z.  Every text row's cosine is the reference's apDot
// (fp64, summed in index order by one thread per row) rounded to float; the per-label maximum
// is an order-free float max (compare-and-swap loop in shared memory); the log-sigmoid and the
// log-sum-exp normalisation run in label order on one thread, as the reference does.
// k_name: one warp per object; the per-label log posteriors are computed lane-parallel, the
// softmax sums, the first-maximum search and the hypernym roll-up in label order on lane 0.
// Device exp/log/log1p may differ from the host libm in the last bit, so log-likelihoods and
// posteriors match the reference to ~1e-7 relative, not bit for bit.
#pragma once
#include "dev_util.cuh"

#define TXT_MAX_LABELS 1024


// apLabelLogLik of one embedding zs (shared memory, T.dim floats) into out[T.n_labels]; best:
// T.n_labels floats of shared scratch.  All threads of the block call it; it ends with a barrier.
DEV void label_loglik_block(const TextDev& T, const float* zs, float* best, float* out) {
  const int tid = threadIdx.x;
  for (int l = tid; l < T.n_labels; l += blockDim.x) best[l] = -2.f;
  __syncthreads();
  for (int r = tid; r < T.rows; r += blockDim.x) {
    const int l = T.row_label[r];
    if (l < 0 || l >= T.n_labels) continue;
    const float* a = T.text + (size_t)r * T.dim;
    double s = 0;
    for (int k = 0; k < T.dim; ++k) s += (double)a[k] * (double)zs[k];   // apDot (objprob.cpp:215-219)
    const float c = (float)s;
    // float max by compare-and-swap (cosines and the -2 start value are finite)
    float old = best[l];
    while (c > old) {
      const float prev = __int_as_float(atomicCAS((int*)&best[l], __float_as_int(old), __float_as_int(c)));
      if (prev == old) break;
      old = prev;
    }
  }
  __syncthreads();
  if (tid == 0) {
    double mx = -1e300;
    for (int l = 0; l < T.n_labels; ++l) {
      out[l] = -1e30f;
      if (best[l] < -1.5f) continue;
      const double x = (double)best[l] * (double)T.scale + (double)T.bias;
      const double ls = x >= 0 ? -log1p(exp(-x)) : x - log1p(exp(x));
      out[l] = (float)ls;
      mx = smax(mx, ls);
    }
    double se = 0;
    for (int l = 0; l < T.n_labels; ++l)
      if (out[l] > -1e29f) se += exp((double)out[l] - mx);
    const double lz = mx + log(smax(se, 1e-300));
    for (int l = 0; l < T.n_labels; ++l)
      if (out[l] > -1e29f) out[l] = (float)((double)out[l] - lz);
  }
  __syncthreads();
}

__global__ void __launch_bounds__(256) k_label_loglik(TextDev T, const float* z, int n, float* out) {
  extern __shared__ __align__(16) unsigned char tx_raw[];
  float* zs = (float*)tx_raw;
  float* best = zs + T.dim;   // per label: max cosine (float)
  const int i = blockIdx.x, tid = threadIdx.x;
  if (i >= n) return;
  for (int k = tid; k < T.dim; k += blockDim.x) zs[k] = z[(size_t)i * T.dim + k];
  __syncthreads();
  label_loglik_block(T, zs, best, out + (size_t)i * T.n_labels);
}

struct NameArgs {
  int n_obj;
  double whole_w, name_wmax, size_w, name_tau;
  const float* L_frag;   // n_obj x C or null
  const double* lw_frag;
  const float* L_whole;  // n_obj x C or null
  const double* lw_whole;
  const float* L_ext;    // n_obj x C or null
  const float* L_geo;    // n_obj x C or null
  const double* size;    // n_obj
  float* post;           // n_obj x C
  int32_t* lab;          // n_obj x 3: name_lab, top_lab, rolled (name_lab -2: no name produced)
  float* val;            // n_obj x 3: name_p, top_p, name_H
};

__global__ void __launch_bounds__(256) k_name(TextDev T, NameArgs a) {
  extern __shared__ __align__(16) unsigned char nm_raw[];
  const int C = T.n_labels, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int o = blockIdx.x * (blockDim.x >> 5) + wid;
  if (o >= a.n_obj) return;
  double* lp = (double*)nm_raw + (size_t)wid * 2 * C;   // C log posteriors, then C doubles of scratch
  double* up = lp + C;
  float* post = a.post + (size_t)o * C;
  const size_t b = (size_t)o * C;
  // lw (apName: fragments, then whole views weighted whole_w)
  double lw = 0;
  if (a.L_frag) lw += a.lw_frag[o];
  if (a.L_whole) lw += a.whole_w * a.lw_whole[o];
  if (!(lw > 0)) {
    if (lane == 0) a.lab[3 * o] = -2;
    return;
  }
  const double lam = lw > a.name_wmax ? a.name_wmax / lw : 1.0;   // name_lambda
  const double ls = log(smax(a.size[o], 0.02));
  for (int c = lane; c < C; c += 32) {
    float L = 0.f;
    if (a.L_frag) L += a.L_frag[b + c];
    if (a.L_whole) L += (float)(a.whole_w * (double)a.L_whole[b + c]);
    double v = lam * (double)L;
    if (L < -1e29f || (double)L <= -60.0 * lw) v = -1e300;
    if (T.log_prior) v += (double)T.log_prior[c];
    if (a.L_ext) v += (double)a.L_ext[b + c];
    if (a.L_geo) v += (double)a.L_geo[b + c];
    if (T.ls_sd && T.ls_sd[c] > 0) {
      const double zz = (ls - (double)T.ls_mu[c]) / (double)T.ls_sd[c];
      v += a.size_w * (-0.5 * zz * zz - log((double)T.ls_sd[c]));
    }
    lp[c] = v;
  }
  __syncwarp();
  if (lane != 0) return;
  // softmax_post (objprob_math.h:102-120), dead = -1e299, no rest group
  const double dead = -1e299;
  double mx = dead;
  bool any = false;
  for (int c = 0; c < C; ++c)
    if (lp[c] > dead) { mx = any ? smax(mx, lp[c]) : lp[c]; any = true; }
  double se = 0;
  for (int c = 0; c < C; ++c)
    if (lp[c] > dead) se += exp(lp[c] - mx);
  se += 0.0;
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
  if (best >= 0 && (double)top_p >= a.name_tau) {
    name_lab = best;
    name_p = top_p;
  } else {
    // hypernym roll-up: probability under each ancestor (8 levels), the deepest one >= name_tau
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
      if (up[c] >= a.name_tau && (gsel < 0 || dpt > gdep || (dpt == gdep && up[c] > ug))) { gsel = c; gdep = dpt; }
    }
    rolled = 1;
    if (gsel >= 0) { name_lab = gsel; name_p = (float)up[gsel]; }
    else if (T.object_label >= 0) { name_lab = T.object_label; name_p = top_p; }
    else { name_lab = best; name_p = top_p; rolled = 0; }
  }
  a.lab[3 * o] = name_lab;
  a.lab[3 * o + 1] = best;
  a.lab[3 * o + 2] = rolled;
  a.val[3 * o] = name_p;
  a.val[3 * o + 1] = top_p;
  a.val[3 * o + 2] = (float)H;
}
