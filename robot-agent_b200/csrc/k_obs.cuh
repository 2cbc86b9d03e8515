// Observation build: one CTA per (detection, map).
//
// Restates scenemap src/objmap.cpp:645-765 (per-detection back-projection, MAD depth band,
// per-observation voxel de-duplication, 10/50/90 percentile boxes, view kappa) and the plane
// fit of apObsStructural (objmap.cpp:565-575 -> apPlaneFit, objprob.cpp:130-209).  The final,
// order-dependent structural decision (ceiling estimate) is taken by k_obs_finalize in
// detection order.
//
// Device data flow per CTA: the box is scanned at stride sk in raster order; valid pixels are
// compacted in raster order (block scan) into L2-resident scratch; every order-sensitive rule of
// the reference (subsample v[(i*n)/2048], first point per voxel, percentiles) is applied to that
// raster-ordered list, and percentiles are exact k-th order statistics (radix selection).
#pragma once
#include "dev_util.cuh"

#define OBS_THREADS 512
#define OBS_HASH 8192
#define OBS_SMEM (OBS_HASH * 12)   // k_obs dynamic shared memory: the voxel hash, reused by later phases
static_assert(3 * SMG_SUB * 8 + SEL_HIST(9) * 4 + 9 * SEL_LIST * 8 <= OBS_SMEM,
              "k_obs: the percentile subsamples, histograms and candidate lists must fit the hash's shared memory");
#define OBS_PPT 4      // raster pixels per thread in the back-projection
#define RANSAC_MAX 256
#define RANSAC_DRAWS (3 * RANSAC_MAX + 64)
#define RANSAC_DBUF (2 * RANSAC_DRAWS)   // draw buffer a caller of plane_fit provides (ints)
// nsamp = ceil(n / max(1, n / min(n, 256))) <= 511, and cnt <= nsamp (objprob.cpp:135-158)
#define NEED_N 512

// Shared-memory working set of plane_fit, provided by the caller (a kernel whose dynamic
// shared memory is free at that point passes a slice of it).
struct PlaneSmem {
  double pl[RANSAC_MAX][4];   // hypothesis planes
  int hist[SEL_HIST(SEL_MAXQ)];   // selection histograms
  int draws[RANSAC_DBUF];     // RANSAC draws + next-triple table
  int id[RANSAC_MAX][3];      // hypothesis index triples
  int cnt[RANSAC_MAX];        // hypothesis inlier counts
};

struct PlaneOut {
  int ok;
  double n[3], thick, inl, zmed, zlo, zhi, hspan;
};

// cos and sin of th = atan2(y, x) / 2, th in (-pi/2, pi/2], from the half-angle identities
// (cos 2th = x / r, sin 2th = y / r, r = |(x, y)|): the larger of the two comes from its square
// root and the other from sin 2th = 2 s c, so both keep full relative precision (within 2 ulps
// of cos/sin of the libm angle).  Reciprocal square roots keep the dependent chain short.
DEV void jacobi_cs(double y, double x, double* c, double* s) {
  const double r2 = x * x + y * y;
  if (!(r2 > 0)) { *c = 1.0; *s = 0.0; return; }
  const double ri = rsqrt(r2);
  if (x >= 0) {
    const double t = 0.5 + 0.5 * (x * ri), rt = rsqrt(t);
    *c = t * rt;
    *s = (0.5 * y * ri) * rt;
  } else {
    const double t = 0.5 - 0.5 * (x * ri), rt = rsqrt(t);
    *s = copysign(t * rt, y);
    *c = (0.5 * y * ri) * copysign(rt, y);
  }
}

// one Jacobi rotation in the (p, q) plane: A <- R^T A R, V <- V R (indices fixed at compile
// time so A and V stay in registers)
template <int p, int q>
DEV void jacobi_rot(double (&A)[3][3], double (&V)[3][3], double c, double s) {
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const double akp = A[k][p], akq = A[k][q];
    A[k][p] = c * akp - s * akq;
    A[k][q] = s * akp + c * akq;
  }
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const double apk = A[p][k], aqk = A[q][k];
    A[p][k] = c * apk - s * aqk;
    A[q][k] = s * apk + c * aqk;
  }
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const double vkp = V[k][p], vkq = V[k][q];
    V[k][p] = c * vkp - s * vkq;
    V[k][q] = s * vkp + c * vkq;
  }
}

// 3x3 symmetric Jacobi eigen-decomposition (scenemap objprob.cpp:50-84): ascending ev, columns V.
// Each step rotates away the largest off-diagonal entry (first of (0,1), (0,2), (1,2) on ties)
// until it is below 1e-12, at most 32 steps.
DEV void eig_sym3(double A[3][3], double ev[3], double V[3][3]) {
  double a[3][3], v[3][3];
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) { a[i][j] = A[i][j]; v[i][j] = i == j; }
  for (int it = 0; it < 32; ++it) {
    int sel = 0;
    double best = fabs(a[0][1]);
    if (fabs(a[0][2]) > best) { best = fabs(a[0][2]); sel = 1; }
    if (fabs(a[1][2]) > best) { best = fabs(a[1][2]); sel = 2; }
    if (best < 1e-12) break;
    double c, s;
    if (sel == 0) { jacobi_cs(2 * a[0][1], a[1][1] - a[0][0], &c, &s); jacobi_rot<0, 1>(a, v, c, s); }
    else if (sel == 1) { jacobi_cs(2 * a[0][2], a[2][2] - a[0][0], &c, &s); jacobi_rot<0, 2>(a, v, c, s); }
    else { jacobi_cs(2 * a[1][2], a[2][2] - a[1][1], &c, &s); jacobi_rot<1, 2>(a, v, c, s); }
  }
  // stable ascending order of the diagonal (insertion sort, like std::sort on 3 elements)
  const double d[3] = {a[0][0], a[1][1], a[2][2]};
  int o0 = 0, o1 = 1, o2 = 2;
  if (d[o1] < d[o0]) { const int t = o0; o0 = o1; o1 = t; }
  if (d[o2] < d[o1]) {
    const int t = o1; o1 = o2; o2 = t;
    if (d[o1] < d[o0]) { const int u = o0; o0 = o1; o1 = u; }
  }
  const int o[3] = {o0, o1, o2};
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    ev[k] = o[k] == 0 ? d[0] : (o[k] == 1 ? d[1] : d[2]);
#pragma unroll
    for (int i = 0; i < 3; ++i) V[i][k] = o[k] == 0 ? v[i][0] : (o[k] == 1 ? v[i][1] : v[i][2]);
  }
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) A[i][j] = a[i][j];
}

DEV int pct_index(int n, double q) {   // min(n-1, size_t(q*(n-1) + 0.5)) (objmap.cpp:17, objprob.cpp:87)
  const int k = (int)(q * (double)(n - 1) + 0.5);
  return k < n - 1 ? k : n - 1;
}

// apPlaneFit (scenemap objprob.cpp:130-209).  xyz: n float points (global).  scr: 4*cap doubles
// of scratch.  The RANSAC iterations run on warp 0 in the reference's sequence (same splitmix
// draws, same adaptive stop; the stop count comes from a host-libm table).  Inlier sums are
// block reductions (deterministic tree).  span1/span2 are not produced (no caller reads them).
DEV void plane_fit(const float* xyz, int n, double tau, uint64_t seed, int max_iters, const int32_t* need_tab, double* scr, int cap,
                   PlaneSmem* ps, BlockScratch& bs, PlaneOut* out, int pbase = 8) {
  PHASE_START();
  __shared__ double sh_best[4];
  __shared__ int sh_bestc;
  __shared__ double sh_m[3], sh_V[3][3], sh_ev[3];
  __shared__ double red[6 * 32];
  const int tid = threadIdx.x;
  if (n < 8 || !(tau > 0)) {
    if (tid == 0) out->ok = 0;
    __syncthreads();
    return;
  }
  // RANSAC (objprob.cpp:133-163).  The index triples do not depend on the inlier counts, so
  // thread 0 draws all of them in the reference's splitmix sequence, every warp scores
  // hypotheses in parallel, and thread 0 replays the sequential best/adaptive-stop logic.
  int (*h_id)[3] = ps->id;
  int* h_cnt = ps->cnt;
  double (*h_pl)[4] = ps->pl;
  int* h_draw = ps->draws;
  int* hist = ps->hist;
  const int iters = max_iters < RANSAC_MAX ? max_iters : RANSAC_MAX;
  const int ns = n < 256 ? n : 256;
  const int sstep = n / ns > 1 ? n / ns : 1;
  const int nsamp = (n + sstep - 1) / sstep;
  // The splitmix state only advances by a constant, so draw k is mix(rs0 + (k + 1) * gamma):
  // all draws (and their 64-bit remainders, the expensive part) are computed in parallel, and
  // thread 0 then walks them with the reference's rejections (objprob.cpp:140-142), falling
  // back to drawing in sequence if the rejections outrun the precomputed draws.
  const uint64_t rs0 = seed ^ ((uint64_t)n << 32);
  const int ndraw = 3 * iters + 64 < RANSAC_DRAWS ? 3 * iters + 64 : RANSAC_DRAWS;
  int* h_qr = h_draw + RANSAC_DRAWS;
  __shared__ int sh_fb;   // first iteration whose triple is not the next three draws
  if (tid == 0) sh_fb = iters;
  for (int k = tid; k < ndraw; k += blockDim.x) {
    uint64_t s = rs0 + (uint64_t)k * 0x9E3779B97F4A7C15ull;
    h_draw[k] = (int)(splitmix(s) % (uint64_t)n);
  }
  __syncthreads();
  // For every start position p: the positions q, r of the second and third index the
  // reference's rejection loops take from there (packed q | r << 16; -1 past the precomputed
  // draws).  Iterations before the first rejection are filled in parallel; from there the
  // walk is one dependent load per iteration.
  for (int p = tid; p < ndraw; p += blockDim.x) {
    const int i0 = h_draw[p];
    int q = p + 1;
    while (q < ndraw && h_draw[q] == i0) ++q;
    int r = q + 1;
    while (r < ndraw && (h_draw[r] == i0 || h_draw[r] == h_draw[q])) ++r;
    h_qr[p] = r < ndraw ? q | (r << 16) : -1;
    if (p % 3 == 0 && p / 3 < iters && !(q == p + 1 && r == p + 2 && r < ndraw)) atomicMin(&sh_fb, p / 3);
  }
  __syncthreads();
  // until the first rejection, iteration it draws positions 3it, 3it+1, 3it+2
  const int fb = sh_fb;
  for (int it = tid; it < fb; it += blockDim.x) {
    h_id[it][0] = h_draw[3 * it]; h_id[it][1] = h_draw[3 * it + 1]; h_id[it][2] = h_draw[3 * it + 2];
  }
  if (tid == 0) {
    int pos = 3 * fb, it = fb;
    for (; it < iters && pos < ndraw; ++it) {
      const int e = h_qr[pos];
      if (e < 0) break;
      h_id[it][0] = h_draw[pos]; h_id[it][1] = h_draw[e & 0xffff]; h_id[it][2] = h_draw[e >> 16];
      pos = (e >> 16) + 1;
    }
    uint64_t rs = rs0;
    auto draw = [&]() -> int {   // the rest in sequence: precomputed draws, then fresh ones
      if (pos < ndraw) { ++pos; return h_draw[pos - 1]; }
      if (pos == ndraw) rs = rs0 + (uint64_t)ndraw * 0x9E3779B97F4A7C15ull;
      ++pos;
      return (int)(splitmix(rs) % (uint64_t)n);
    };
    for (; it < iters; ++it) {
      const int id0 = draw();
      int id1, id2;
      do id1 = draw(); while (id1 == id0);
      do id2 = draw(); while (id2 == id0 || id2 == id1);
      h_id[it][0] = id0; h_id[it][1] = id1; h_id[it][2] = id2;
    }
  }
  __syncthreads();
  // Score the hypotheses a warp each, one batch of (warps) at a time; after each batch thread 0
  // continues the reference's walk (best so far, adaptive stop) over the newly scored ones, and
  // the scoring ends as soon as the walk has ended: later hypotheses would never be looked at.
  __shared__ int sh_more;
  if (tid == 0) sh_bestc = -1;
  double best[4] = {0, 0, 1, 0};
  int best_c = -1, need = max_iters > 1 ? max_iters : 1, walk = 0;   // thread 0's walk state
  const int lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
  for (int r0 = 0; r0 < iters; r0 += nw) {
    const int it = r0 + wid;
    if (it < iters) {
      if (!INB(h_id[it][0], n, 105) || !INB(h_id[it][1], n, 105) || !INB(h_id[it][2], n, 105)) {
        if (lane == 0) h_cnt[it] = -1;
      } else {
        const float* a = xyz + 3 * h_id[it][0];
        const float* b = xyz + 3 * h_id[it][1];
        const float* c = xyz + 3 * h_id[it][2];
        const double u[3] = {(double)(b[0] - a[0]), (double)(b[1] - a[1]), (double)(b[2] - a[2])};
        const double v[3] = {(double)(c[0] - a[0]), (double)(c[1] - a[1]), (double)(c[2] - a[2])};
        double nn[3] = {u[1] * v[2] - u[2] * v[1], u[2] * v[0] - u[0] * v[2], u[0] * v[1] - u[1] * v[0]};
        const double L = sqrt(nn[0] * nn[0] + nn[1] * nn[1] + nn[2] * nn[2]);
        if (L < 1e-6) {   // nearly collinear: the reference skips the iteration
          if (lane == 0) h_cnt[it] = -1;
        } else {
          for (int k = 0; k < 3; ++k) nn[k] /= L;
          const double d0 = -(nn[0] * (double)a[0] + nn[1] * (double)a[1] + nn[2] * (double)a[2]);
          int cnt = 0;
          for (int s = lane; s < nsamp; s += 32) {
            const int i = s * sstep;
            if (!INB(i, n, 119)) break;
            cnt += fabs(nn[0] * (double)xyz[3 * i] + nn[1] * (double)xyz[3 * i + 1] + nn[2] * (double)xyz[3 * i + 2] + d0) <= tau;
          }
          cnt = warp_sum_i(cnt);
          if (lane == 0) {
            h_cnt[it] = cnt;
            h_pl[it][0] = nn[0]; h_pl[it][1] = nn[1]; h_pl[it][2] = nn[2]; h_pl[it][3] = d0;
          }
        }
      }
    }
    __syncthreads();
    if (tid == 0) {
      const int end = r0 + nw < iters ? r0 + nw : iters;
      bool stop = false;
      for (; walk < need && walk < end; ++walk) {
        const int cnt = h_cnt[walk];
        if (cnt < 0) continue;
        if (cnt > best_c) {
          best_c = cnt;
          for (int k = 0; k < 4; ++k) best[k] = h_pl[walk][k];
          const double w = (double)cnt / (double)nsamp;
          const double pw = w * w * w;
          if (pw > 0.999999) { stop = true; break; }
          if (pw > 1e-9 && INB(nsamp * NEED_N + cnt, NEED_N * NEED_N, 120)) need = need_tab[nsamp * NEED_N + cnt];
        }
      }
      sh_more = !stop && walk < need && walk < iters;
      if (!sh_more) {
        sh_bestc = best_c;
        for (int k = 0; k < 4; ++k) sh_best[k] = best[k];
      }
    }
    __syncthreads();
    if (!sh_more) break;
  }
  __syncthreads();
  if (sh_bestc < 3) {
    if (tid == 0) out->ok = 0;
    __syncthreads();
    return;
  }
  PHASE_MARK(pbase + 0);   // RANSAC
  // two PCA refits (objprob.cpp:166-180); mp = plane whose inliers the last pass used.
  // Sums are block trees.  Where the outcome is ill-conditioned in the reference's own rounding
  // (a point within 1e-11 of the tau boundary, a near-double smallest eigenvalue, a nearly
  // isotropic horizontal spread), thread 0 replays the whole refit with the reference's
  // sequential sums in index order, so inlier sets and sums are the reference's (the Jacobi
  // rotations come from half-angle identities, within a few ulps of libm's trigonometry).  A near-zero
  // smallest eigenvalue (exactly planar points) is well-conditioned for the normal; only the
  // thickness sqrt(ev0) then differs, by at most ~sqrt(1e-16 * ev2).
  __shared__ int sh_deg, sh_ni, sh_ok;
  __shared__ double sh_mp[4], sh_hc, sh_hs;
  if (tid == 0) sh_deg = 0;
  double pl[4] = {sh_best[0], sh_best[1], sh_best[2], sh_best[3]};
  double mp[4];
  double ch[3] = {0, 0, 0};   // the last pass's horizontal second moments (c00, c01, c11)
  int ni = 0;
  for (int pass = 0; pass < 2; ++pass) {
    for (int k = 0; k < 4; ++k) mp[k] = pl[k];
    double sm[5] = {0, 0, 0, 0, 0};   // count, sum x, sum y, sum z, near-boundary points
    for (int i = tid; i < n; i += blockDim.x) {
      const double x = xyz[3 * i], y = xyz[3 * i + 1], z = xyz[3 * i + 2];
      const double dd = fabs(mp[0] * x + mp[1] * y + mp[2] * z + mp[3]);
      if (dd <= tau) { sm[0] += 1.0; sm[1] += x; sm[2] += y; sm[3] += z; }
      if (fabs(dd - tau) <= 1e-11) sm[4] += 1.0;
    }
    block_sum_multi<5>(sm, red);
    ni = (int)sm[0];
    if (sm[4] > 0 && tid == 0) sh_deg = 1;
    if (ni < 3) break;
    const double inv = 1.0 / (double)(ni > 1 ? ni : 1);
    double m[3] = {sm[1], sm[2], sm[3]};
    for (int k = 0; k < 3; ++k) m[k] *= inv;
    double c[6] = {0, 0, 0, 0, 0, 0};
    for (int i = tid; i < n; i += blockDim.x) {
      const double x = xyz[3 * i], y = xyz[3 * i + 1], z = xyz[3 * i + 2];
      if (fabs(mp[0] * x + mp[1] * y + mp[2] * z + mp[3]) <= tau) {
        const double d[3] = {x - m[0], y - m[1], z - m[2]};
        c[0] += d[0] * d[0]; c[1] += d[0] * d[1]; c[2] += d[0] * d[2];
        c[3] += d[1] * d[1]; c[4] += d[1] * d[2]; c[5] += d[2] * d[2];
      }
    }
    block_sum_multi<6>(c, red);
    ch[0] = c[0]; ch[1] = c[1]; ch[2] = c[3];
    double C[3][3];
    C[0][0] = c[0] * inv; C[0][1] = c[1] * inv; C[0][2] = c[2] * inv;
    C[1][1] = c[3] * inv; C[1][2] = c[4] * inv; C[2][2] = c[5] * inv;
    C[1][0] = C[0][1]; C[2][0] = C[0][2]; C[2][1] = C[1][2];
    if (tid == 0) {
      double ev[3], V[3][3];
      eig_sym3(C, ev, V);
      for (int i = 0; i < 3; ++i) {
        sh_ev[i] = ev[i];
        sh_m[i] = m[i];
        for (int j = 0; j < 3; ++j) sh_V[i][j] = V[i][j];
      }
      if (ev[1] - ev[0] <= 1e-3 * ev[2]) sh_deg = 1;   // near-double smallest eigenvalue: the normal is ill-defined
    }
    __syncthreads();
    pl[0] = sh_V[0][0]; pl[1] = sh_V[1][0]; pl[2] = sh_V[2][0];
    pl[3] = -(pl[0] * sh_m[0] + pl[1] * sh_m[1] + pl[2] * sh_m[2]);
  }
  double th_hc = 0, th_hs = 0;
  if (ni >= 3) {
    // horizontal principal direction of the inliers (objprob.cpp:187-192): its sums over the
    // last pass's inliers about the last pass's mean are that pass's covariance sums c00, c01,
    // c11 (the same points, the same operations, the same reduction tree)
    const double sxx = ch[0], sxy = ch[1], syy = ch[2];
    if (tid == 0 && 2 * fabs(sxy) + fabs(sxx - syy) <= 1e-3 * (sxx + syy)) sh_deg = 1;
    jacobi_cs(2 * sxy, sxx - syy, &th_hc, &th_hs);
  }
  __syncthreads();
  PHASE_MARK(pbase + 1);   // PCA refits (parallel)
  if (sh_deg) {   // exact replay in the reference's order (pcaOf objprob.cpp:101-114, :166-192)
    if (tid == 0) {
      double q[4] = {sh_best[0], sh_best[1], sh_best[2], sh_best[3]}, qm[4] = {0, 0, 0, 0};
      double m[3] = {0, 0, 0}, ev[3] = {0, 0, 0}, V[3][3];
      int nin = 0;
      for (int pass = 0; pass < 2 && (pass == 0 || nin >= 3); ++pass) {
        for (int k = 0; k < 4; ++k) qm[k] = q[k];
        nin = 0;
        m[0] = m[1] = m[2] = 0;
        for (int i = 0; i < n; ++i)
          if (fabs(qm[0] * xyz[3 * i] + qm[1] * xyz[3 * i + 1] + qm[2] * xyz[3 * i + 2] + qm[3]) <= tau) {
            ++nin;
            for (int k = 0; k < 3; ++k) m[k] += xyz[3 * i + k];
          }
        if (nin < 3) break;
        const double inv = 1.0 / (double)(nin > 1 ? nin : 1);
        for (int k = 0; k < 3; ++k) m[k] *= inv;
        double C[3][3] = {{0, 0, 0}, {0, 0, 0}, {0, 0, 0}};
        for (int i = 0; i < n; ++i)
          if (fabs(qm[0] * xyz[3 * i] + qm[1] * xyz[3 * i + 1] + qm[2] * xyz[3 * i + 2] + qm[3]) <= tau) {
            const double d[3] = {xyz[3 * i] - m[0], xyz[3 * i + 1] - m[1], xyz[3 * i + 2] - m[2]};
            for (int r = 0; r < 3; ++r)
              for (int cc = 0; cc < 3; ++cc) C[r][cc] += d[r] * d[cc];
          }
        for (int r = 0; r < 3; ++r)
          for (int cc = 0; cc < 3; ++cc) C[r][cc] *= inv;
        eig_sym3(C, ev, V);
        q[0] = V[0][0]; q[1] = V[1][0]; q[2] = V[2][0];
        q[3] = -(q[0] * m[0] + q[1] * m[1] + q[2] * m[2]);
      }
      sh_ok = nin >= 3;
      sh_ni = nin;
      if (nin >= 3) {
        double sxx = 0, sxy = 0, syy = 0;
        for (int i = 0; i < n; ++i)
          if (fabs(qm[0] * xyz[3 * i] + qm[1] * xyz[3 * i + 1] + qm[2] * xyz[3 * i + 2] + qm[3]) <= tau) {
            const double dx = xyz[3 * i] - m[0], dy = xyz[3 * i + 1] - m[1];
            sxx += dx * dx; sxy += dx * dy; syy += dy * dy;
          }
        double hc, hs;
        jacobi_cs(2 * sxy, sxx - syy, &hc, &hs);
        sh_hc = hc;
        sh_hs = hs;
        for (int i = 0; i < 3; ++i) {
          sh_ev[i] = ev[i];
          sh_m[i] = m[i];
          for (int j = 0; j < 3; ++j) sh_V[i][j] = V[i][j];
        }
        for (int k = 0; k < 4; ++k) sh_mp[k] = qm[k];
      }
    }
    __syncthreads();
    if (!sh_ok) {
      if (tid == 0) out->ok = 0;
      __syncthreads();
      return;
    }
    ni = sh_ni;
    for (int k = 0; k < 4; ++k) mp[k] = sh_mp[k];
    th_hc = sh_hc;
    th_hs = sh_hs;
  } else if (ni < 3) {
    if (tid == 0) out->ok = 0;
    __syncthreads();
    return;
  }
  const double m0 = sh_m[0], m1 = sh_m[1], hc = th_hc, hs = th_hs;
  if (sh_deg) PHASE_MARK(pbase + 3);   // sequential replay (only when it ran)
  // z and horizontal-span projections of the inliers -> exact percentiles (objprob.cpp:193-206)
  __shared__ int sh_cnt;
  if (tid == 0) sh_cnt = 0;
  __syncthreads();
  double* zs = scr;
  double* hsp = scr + cap;
  for (int i = tid; i < n; i += blockDim.x) {
    const double x = xyz[3 * i], y = xyz[3 * i + 1], z = xyz[3 * i + 2];
    if (fabs(mp[0] * x + mp[1] * y + mp[2] * z + mp[3]) <= tau) {
      const int q = atomicAdd(&sh_cnt, 1);
      if (!INB(q, cap, 104)) continue;
      zs[q] = z;
      hsp[q] = (x - m0) * hc + (y - m1) * hs;
    }
  }
  __syncthreads();
  __shared__ double sel5[5];
  {
    const double* arr[5] = {hsp, hsp, zs, zs, zs};
    const int nn[5] = {ni, ni, ni, ni, ni};
    const int kk[5] = {pct_index(ni, 0.9), pct_index(ni, 0.1), pct_index(ni, 0.1), pct_index(ni, 0.9), pct_index(ni, 0.5)};
    block_select_multi(arr, nn, kk, sel5, 5, hist, bs);
  }
  const double h9 = sel5[0], h1 = sel5[1], zlo = sel5[2], zhi = sel5[3], zmd = sel5[4];
  if (tid == 0) {
    out->ok = 1;
    for (int k = 0; k < 3; ++k) out->n[k] = sh_V[k][0];
    out->thick = sqrt(smax(0.0, sh_ev[0]));
    out->inl = (double)ni / (double)n;
    out->hspan = h9 - h1;
    out->zlo = zlo;
    out->zhi = zhi;
    out->zmed = zmd;
  }
  __syncthreads();
  PHASE_MARK(pbase + 2);   // percentiles
}

// subsample (objmap.cpp:37-42) of v[0..n) into S (<= SMG_SUB values); returns its size.
// Each thread issues its (up to 4) loads before storing any.  No barrier: the caller syncs.
// A point of the back-projection is kept as its pixel (v << 16 | u) and float depth; its map
// coordinates are recomputed where needed with the same operations (objmap.cpp:680-683), so
// every use sees the same doubles the reference computes, and the per-point scratch traffic is
// 8 bytes instead of 40.
DEV void bp_map(const FrameDev& F, uint32_t pix, float z, double* X, double* Y, double* Zm) {
  const int uu = (int)(pix & 0xffffu), vv = (int)(pix >> 16);
  const double xc = (double)(((float)uu - F.cx) / F.fx * z), yc = (double)(((float)vv - F.cy) / F.fy * z);
  const double zd = (double)z;
  const double* T = F.T_mc;
  *X = T[0] * xc + T[1] * yc + T[2] * zd + T[3];
  *Y = T[4] * xc + T[5] * yc + T[6] * zd + T[7];
  *Zm = T[8] * xc + T[9] * yc + T[10] * zd + T[11];
}

// the detector-image pixel a point's mask cell is read at (objmap.cpp:686-687)
DEV void bp_cell(const FrameDev& F, uint32_t pix, bool bits_form, int32_t* pu, int32_t* pv) {
  const int uu = (int)(pix & 0xffffu), vv = (int)(pix >> 16);
  if (bits_form) {
    *pu = (int)(((float)uu + 0.5f) / F.sxu_f);
    *pv = (int)(((float)vv + 0.5f) / F.syv_f);
  } else {
    *pu = uu;
    *pv = vv;
  }
}

// subsample_to of the depths (double) of the float depth list
DEV int subsample_z(const float* v, int n, double* S) {
  const int nS = n <= SMG_SUB ? n : SMG_SUB;
  for (int i = threadIdx.x; i < nS; i += blockDim.x) {
    const size_t src = n <= SMG_SUB ? (size_t)i : (size_t)i * (size_t)n / SMG_SUB;
    S[i] = INB(src, n, 118) ? (double)v[src] : 0.0;
  }
  return nS;
}

// the three coordinate subsamples of the kept points (indices KI into the point list)
DEV int subsample_xyz(const FrameDev& F, const uint32_t* PIX, const float* ZF, const int32_t* KI, int np, int n, double* SX,
                      double* SY, double* SZ) {
  const int nS = np <= SMG_SUB ? np : SMG_SUB;
  for (int i = threadIdx.x; i < nS; i += blockDim.x) {
    const size_t src = np <= SMG_SUB ? (size_t)i : (size_t)i * (size_t)np / SMG_SUB;
    double x = 0, y = 0, z = 0;
    if (INB(src, np, 121)) {
      const int p = KI[src];
      if (INB(p, n, 122)) bp_map(F, PIX[p], ZF[p], &x, &y, &z);
    }
    SX[i] = x; SY[i] = y; SZ[i] = z;
  }
  return nS;
}

DEV int subsample_to(const double* v, int n, double* S) {
  const int nS = n <= SMG_SUB ? n : SMG_SUB;
  for (int c0 = 0; c0 < nS; c0 += 4 * blockDim.x) {
    double t[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = c0 + j * blockDim.x + threadIdx.x;
      const size_t src = n <= SMG_SUB ? (size_t)i : (size_t)i * (size_t)n / SMG_SUB;
      t[j] = i < nS && INB(src, n, 118) ? v[src] : 0.0;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = c0 + j * blockDim.x + threadIdx.x;
      if (i < nS && INB(i, SMG_SUB, 117)) S[i] = t[j];
    }
  }
  return nS;
}


__global__ void __launch_bounds__(OBS_THREADS, 2) k_obs(Batch B) {   // 2 CTAs per SM: <= 64 registers
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* hkey = (uint64_t*)smem_raw;                         // OBS_HASH keys
  uint32_t* hidx = (uint32_t*)(smem_raw + OBS_HASH * 8);        // OBS_HASH first index
  double* S = (double*)smem_raw;                                // SMG_SUB values (aliases the hash)
  int* hist = (int*)(S + SMG_SUB);                              // MAD selection histogram
  __shared__ BlockScratch bs;
  __shared__ PlaneOut pout;
  const int m = B.map0 + blockIdx.y, k = blockIdx.x, tid = threadIdx.x;
  const FrameDev& F = B.frames[m];
  ObsRec* O = &B.obs[(size_t)m * B.max_det + k];
  if (tid == 0) {   // no text model / embedding (k_obs_text overwrites these when there is one)
    O->ps = -1.0; O->pso = 0.0; O->top_p = 0.0; O->top_lab = -1; O->so_sh = 1; O->wall_like = 0; O->struct_look = 0;
  }
  if (!F.active || k >= F.n_det) {
    if (tid == 0) { O->valid = 0; O->stage = -1; O->floor_drop = 0; }
    return;
  }
  const smg_params& P = B.p;
  const int W = F.w, H = F.h;
#ifdef SMG_CHECKS
  if (F.depth == nullptr || (F.label == nullptr && F.mask_bits == nullptr) || W <= 0 || H <= 0 || W > B.W || H > B.H || m >= B.M) {
    if (tid == 0) smg_chk_fail(110, (long long)(size_t)F.depth, (long long)(size_t)F.label);
    return;
  }
#endif
  const size_t slot = (size_t)m * B.max_det + k;
  uint32_t* PIX = (uint32_t*)(B.px + slot * 4 * B.pmax);   // per point: pixel (v << 16 | u)
  float* ZF = (float*)(PIX + B.pmax);                       // per point: depth
  int32_t* KI = (int32_t*)(ZF + B.pmax);                    // kept points (band filter), in order
  float* CX = B.cxyz + slot * 3 * B.pmax;
  int32_t* CP = B.cpx + slot * 2 * B.pmax;
  double* SCR = B.sel + slot * 4 * B.pmax;
  const uint16_t L = F.det_label[k];
  const bool bits_form = F.mask_bits != nullptr;
  // box scan (objmap.cpp:648-652): detector box -> depth pixels
  const int st = P.step > 1 ? P.step : 1;
  int u0, u1, v0, v1;
  det_scan_box(F, k, &u0, &u1, &v0, &v1);
  const double box_px = (double)max(0, u1 - u0 + 1) * (double)max(0, v1 - v0 + 1);
  const int sk = max(st, (int)ceil(sqrt(box_px / (double)max(1, P.max_pts))));
  const int ncols = u1 >= u0 ? (u1 - u0) / sk + 1 : 0, nrows = v1 >= v0 ? (v1 - v0) / sk + 1 : 0;
  const int npix = ncols * nrows;
  if (npix > B.pmax) {
    if (tid == 0) { O->valid = 0; O->stage = 0; set_err(&B.maps[m], SMG_E_CAP_PTS); }
    return;
  }
  if (tid == 0) { wk_add(&B.maps[m], SMG_WK_OBS_PX, npix); wk_add(&B.maps[m], SMG_WK_DET, 1); }
  PHASE_START();
  const double* T = F.T_mc;
  __shared__ int scan_db[2][33];
  int scan_it = 0;
  // 1. back-projection in raster order (objmap.cpp:667-688), ordered compaction.  Each thread
  // takes OBS_PPT consecutive raster pixels and issues all their label and depth loads before
  // using any, so one round trip to memory covers them.
  int n = 0;
  for (int c0 = 0; c0 < npix; c0 += blockDim.x * OBS_PPT) {
    const int i0 = c0 + tid * OBS_PPT;
    float zv[OBS_PPT];
    int okm = 0;
#pragma unroll
    for (int j = 0; j < OBS_PPT; ++j) {
      const int idx = i0 + j;
      zv[j] = 0.f;
      if (idx < npix) {
        const int r = idx / ncols, cc = idx - r * ncols;
        const int uu = u0 + cc * sk, vv = v0 + r * sk;
        if (bits_form) {   // the detector's bit masks on their own grid
          int pu, pv;
          if (det_bits_at(F, k, uu, vv, &pu, &pv) && INB((size_t)vv * W + uu, (size_t)W * H, 111)) {
            const float z = F.depth[(size_t)vv * W + uu];
            if (z > P.zmin && z < P.zmax) { okm |= 1 << j; zv[j] = z; }
          }
        } else if (vv >= 1 && vv < H - 1 && INB((size_t)vv * W + uu, (size_t)W * H, 111)) {
          // label image: mask cell (i, j) = pixel (u, v); 1-cell erosion; rows j < 1 or j >= MH-1
          // are skipped
          const size_t at = (size_t)vv * W + uu;
          const uint16_t* lp = F.label + at;
          const bool lm = (lp[0] == L) & (uu > 0 && lp[-1] == L) & (uu + 1 < W && lp[1] == L) & (lp[-W] == L) & (lp[W] == L);
          const float z = F.depth[at];
          if (lm && z > P.zmin && z < P.zmax) { okm |= 1 << j; zv[j] = z; }
        }
      }
    }
    int tot;
    int o = n + block_scan_db(__popc(okm), &tot, scan_db, scan_it++);
#pragma unroll
    for (int j = 0; j < OBS_PPT; ++j) {
      if (!((okm >> j) & 1)) continue;
      const int idx = i0 + j, r = idx / ncols, cc = idx - r * ncols;
      const int uu = u0 + cc * sk, vv = v0 + r * sk;
      if (INB(o, B.pmax, 101)) {
        PIX[o] = (uint32_t)vv << 16 | (uint32_t)uu;
        ZF[o] = zv[j];
      }
      ++o;
    }
    n += tot;
  }
  if (n < P.min_points) {
    if (tid == 0) { O->valid = 0; O->stage = 1; O->floor_drop = 0; }
    return;
  }
  __syncthreads();
  PHASE_MARK(0);   // back-projection
  // 2. MAD depth band (objmap.cpp:692-695)
  int nS = subsample_z(ZF, n, S);
  __syncthreads();
  const int kmed = pct_index(nS, 0.5);
  unsigned long long* slist = (unsigned long long*)(hist + SEL_HIST(1));   // candidate list of the selection
  const double zmed = block_select(S, nS, kmed, hist, bs, slist);
  for (int i = tid; i < nS; i += blockDim.x) S[i] = fabs(S[i] - zmed);
  __syncthreads();
  const double mad = block_select(S, nS, kmed, hist, bs, slist);
  const double band = smax(P.mad_k * 1.4826 * mad, P.mad_floor);
  __syncthreads();
  PHASE_MARK(1);   // MAD band
  // 3. band filter, hand count, first point per voxel (objmap.cpp:696-719)
  for (int i = tid; i < OBS_HASH; i += blockDim.x) { hkey[i] = ~0ull; hidx[i] = 0xffffffffu; }
  __syncthreads();
  const double hand2 = (double)(P.hand_r * P.hand_r), chand2 = P.cloud_hand_r * P.cloud_hand_r, body2 = P.body_r * P.body_r;
  const double* E0 = F.eef[0];
  const double* E1 = F.eef[1];
  int near_local = 0, w = 0;
  int32_t* HS = (int32_t*)SCR;   // per point: its voxel's hash slot, -1 when it enters no voxel
  for (int c0 = 0; c0 < n; c0 += blockDim.x) {
    const int i = c0 + tid;
    int keep = 0, hs = -1;
    if (i < n) {
      keep = INB(i, B.pmax, 112) && !(fabs((double)ZF[i] - zmed) > band);
      if (keep) {
        double x, y, z;
        bp_map(F, PIX[i], ZF[i], &x, &y, &z);
        const double d0 = (x - E0[0]) * (x - E0[0]) + (y - E0[1]) * (y - E0[1]) + (z - E0[2]) * (z - E0[2]);
        const double d1 = (x - E1[0]) * (x - E1[0]) + (y - E1[1]) * (y - E1[1]) + (z - E1[2]) * (z - E1[2]);
        const double dh2 = smin(d0, d1);
        near_local += dh2 < hand2;
        const double bx = x - F.base[0], by = y - F.base[1];
        if (dh2 >= chand2 && bx * bx + by * by >= body2) {
          const uint64_t key = voxel_key((float)x, (float)y, (float)z, B.inv_vox);
          uint32_t h = hmix(key) & (OBS_HASH - 1);
          for (int probe = 0; probe < OBS_HASH; ++probe) {
            const unsigned long long prev = atomicCAS((unsigned long long*)&hkey[h], ~0ull, (unsigned long long)key);
            if (prev == ~0ull || prev == key) { atomicMin(&hidx[h], (uint32_t)i); hs = (int)h; break; }
            h = (h + 1) & (OBS_HASH - 1);
          }
        }
      }
      if (INB(i, B.pmax, 112)) HS[i] = hs;
    }
    int tot;
    const int pos = block_scan_db(keep, &tot, scan_db, scan_it++);
    if (keep && INB(w + pos, B.pmax, 102)) KI[w + pos] = i;
    w += tot;
  }
  const int near_hand = block_sum_i(near_local, bs);
  const int np = w;
  // emit the first point of each voxel, raster order (same thread per point as the pass above)
  int nc = 0;
  for (int c0 = 0; c0 < n; c0 += blockDim.x) {
    const int i = c0 + tid;
    int emit = 0;
    if (i < n && INB(i, B.pmax, 113)) {
      const int hs = HS[i];
      emit = hs >= 0 && INB(hs, OBS_HASH, 114) && hidx[hs] == (uint32_t)i;
    }
    int tot;
    const int pos = block_scan_db(emit, &tot, scan_db, scan_it++);
    if (emit && INB(nc + pos, B.pmax, 103)) {
      double x, y, z;
      bp_map(F, PIX[i], ZF[i], &x, &y, &z);
      CX[3 * (nc + pos)] = (float)x;
      CX[3 * (nc + pos) + 1] = (float)y;
      CX[3 * (nc + pos) + 2] = (float)z;
      bp_cell(F, PIX[i], bits_form, &CP[2 * (nc + pos)], &CP[2 * (nc + pos) + 1]);
    }
    nc += tot;
  }
  if (np < P.min_points || (float)near_hand >= P.hand_frac * (float)np) {
    if (tid == 0) { O->valid = 0; O->stage = 2; O->floor_drop = 0; }
    return;
  }
  __syncthreads();
  PHASE_MARK(2);   // band filter + voxels
  // 4. 10/50/90 percentiles per axis (objmap.cpp:730-738): nine order statistics, one sweep
  double lo[3], md[3], hi[3];
  {
    double* SB[3] = {S, S + SMG_SUB, S + 2 * SMG_SUB};
    int* mh = (int*)(S + 3 * SMG_SUB);
    const int nS3 = subsample_xyz(F, PIX, ZF, KI, np, n, SB[0], SB[1], SB[2]);
    __syncthreads();
    const double* arr[9] = {SB[0], SB[0], SB[0], SB[1], SB[1], SB[1], SB[2], SB[2], SB[2]};
    const int nn[9] = {nS3, nS3, nS3, nS3, nS3, nS3, nS3, nS3, nS3};
    const int kk[9] = {pct_index(nS3, 0.5), pct_index(nS3, 0.1), pct_index(nS3, 0.9), pct_index(nS3, 0.5), pct_index(nS3, 0.1),
                       pct_index(nS3, 0.9), pct_index(nS3, 0.5), pct_index(nS3, 0.1), pct_index(nS3, 0.9)};
    __shared__ double sel9[9];
    block_select_multi(arr, nn, kk, sel9, 9, mh, bs, (unsigned long long*)(mh + SEL_HIST(9)));
    for (int a = 0; a < 3; ++a) { md[a] = sel9[3 * a]; lo[a] = sel9[3 * a + 1]; hi[a] = sel9[3 * a + 2]; }
    __syncthreads();
  }
  const float* b = F.box[k];   // detector-image pixels
  const int trunc = (b[0] <= 2 || b[1] <= 2 || b[2] >= F.img_w - 3 || b[3] >= F.img_h - 3);
  if (tid == 0) {
    O->det = k;
    O->sk = sk;
    O->cls = F.cls[k];
    O->score = F.score[k];
    O->trunc = trunc;
    O->n = np;
    O->nc = nc;
    O->zmed = zmed;
    for (int a = 0; a < 3; ++a) { O->pos[a] = md[a]; O->lo[a] = lo[a]; O->hi[a] = hi[a]; O->ext[a] = hi[a] - lo[a]; }
    O->floor_drop = hi[2] < P.floor_h;   // no floor-level class table: floorLevel() is false
    // viewKappa of a detection fragment (objmap.cpp:757-762, bestview.cpp:77-81)
    const float size_px = (float)sqrt((double)np * sk * sk / smax(1e-9, (double)F.sxu_f * (double)F.syv_f));
    const float depth_m = (float)zmed;
    O->kappa = view_kappa((double)fmaxf(0.f, size_px), trunc, (double)fmaxf(0.f, depth_m), P.kap_k0, P.kap_s0, P.kap_trunc,
                          P.kap_d0, P.kap_occ, P.kap_blur_w, F.blur_fac);
    O->obs_to = -1;
    O->n_same = 0;
    O->blocked = 0;
    O->sec = 0;
  }
  if (hi[2] < P.floor_h) {
    if (tid == 0) { O->valid = 0; O->stage = 3; }
    return;
  }
  PHASE_MARK(3);   // percentiles
  // 5. plane fit of the cloud candidates (apObsStructural, objmap.cpp:565-575)
  double c0s = 0, c1s = 0, c2s = 0;
  for (int i = tid; i < nc && INB(3 * i + 2, 3 * B.pmax, 115); i += blockDim.x) { c0s += CX[3 * i]; c1s += CX[3 * i + 1]; c2s += CX[3 * i + 2]; }
  const double cen0 = block_sum_d(c0s, bs), cen1 = block_sum_d(c1s, bs), cen2 = block_sum_d(c2s, bs);
  if (nc >= 8) {
    const double dc = hypot3(cen0 / nc - T[3], cen1 / nc - T[7], cen2 / nc - T[11]);
    const double tau = smin(P.ransac_tau_max, P.ransac_tau0 + P.ransac_tau_k * dc * dc);
    const uint64_t sb = (uint64_t)__double_as_longlong(F.stamp);
    // the hash is dead: plane-fit working set, then the points when they fit
    PlaneSmem* ps = (PlaneSmem*)smem_raw;
    const float* PX = CX;
    if ((size_t)nc * 12 + sizeof(PlaneSmem) <= OBS_SMEM) {
      float* PXs = (float*)(smem_raw + sizeof(PlaneSmem));
      for (int i = tid; i < 3 * nc; i += blockDim.x) PXs[i] = CX[i];
      __syncthreads();
      PX = PXs;
    }
    PHASE_MARK(4);   // plane-fit set-up
    plane_fit(PX, nc, tau, ap_seed(sb, (uint64_t)k), P.ransac_iters, B.need_tab, SCR, B.pmax, ps, bs, &pout);
  } else if (tid == 0) {
    pout.ok = 0;
  }
  __syncthreads();
  PHASE_MARK(5);
  // wall-line share of apObsStructural (objmap.cpp:606-611): every stp-th candidate, within
  // wall_d of some segment of this keyframe's set
  int w_near = 0, w_tot = 0;
  const int n_wf = B.maps[m].wfr;   // wall segments this keyframe carries
  if (n_wf > 0 && nc >= 8) {
    const double* S = B.wsegs + (size_t)m * SMG_WALL_SEGS_MAX * 4;
    const int stp = nc / 64 > 1 ? nc / 64 : 1;
    w_tot = (nc + stp - 1) / stp;
    int near = 0;
    for (int j = tid; j < w_tot; j += blockDim.x) {
      const int i = j * stp;
      near += wall_dist((double)CX[3 * i], (double)CX[3 * i + 1], S, n_wf, P.wall_d) <= P.wall_d;
    }
    w_near = block_sum_i(near, bs);
  }
  if (tid == 0) {
    O->w_near = w_near;
    O->w_tot = w_tot;
    O->pl_ok = pout.ok;
    for (int a = 0; a < 3; ++a) O->pl_n[a] = pout.n[a];
    O->pl_thick = pout.thick;
    O->pl_inl = pout.inl;
    O->pl_zmed = pout.zmed;
    O->pl_zlo = pout.zlo;
    O->pl_zhi = pout.zhi;
    O->pl_hspan = pout.hspan;
    O->valid = 1;
    O->stage = 4;
  }
}

// Structural decision and observation list, in detection order (objmap.cpp:741-765, the
// see-through drop at :742-753 and the apObsStructural branches at :576-621; ps, pso and the
// shape group come from k_obs_text when a text model is set, the wall-line share from k_obs).
__global__ void k_obs_finalize(Batch B) {
  const int m = B.map0 + blockIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active) return;
  const int n_wf = B.maps[m].wfr;   // wall segments this keyframe carries
  const bool walls = n_wf > 0;
  const double* S = B.wsegs + (size_t)m * SMG_WALL_SEGS_MAX * 4;
  // the fields the decision reads, staged by the warp; the walk then waits on no global load
  struct Fin {
    int valid, stage, nc, pl_ok, so_sh, w_near, w_tot, through;
    double inl, thick, nz, zmed, zhi, zlo, hspan, ps, pso;
  };
  __shared__ Fin fs[SMG_MAX_DET];
  const int nd = min(F.n_det, B.max_det);
  for (int k = threadIdx.x; k < nd; k += blockDim.x) {
    const ObsRec* O = &B.obs[(size_t)m * B.max_det + k];
    Fin f;
    f.valid = O->valid; f.stage = O->stage; f.nc = O->nc; f.pl_ok = O->pl_ok;
    f.inl = O->pl_inl; f.thick = O->pl_thick; f.nz = fabs(O->pl_n[2]); f.zmed = O->pl_zmed;
    f.zhi = O->pl_zhi; f.zlo = O->pl_zlo; f.hspan = O->pl_hspan;
    f.ps = O->ps; f.pso = O->pso; f.so_sh = O->so_sh;
    f.w_near = O->w_near; f.w_tot = O->w_tot;
    // seen through a window (objmap.cpp:742-753): the camera -> centre line crosses a wall
    // segment of this keyframe and the centre lies more than through_d beyond it
    f.through = 0;
    if (O->valid && walls) {
      const double cx0 = F.T_mc[3], cy0 = F.T_mc[7], dx = O->pos[0] - cx0, dy = O->pos[1] - cy0, L = hypot(dx, dy);
      for (int s2 = 0; s2 < n_wf && !f.through && L > 1e-6; ++s2) {
        const double* w = S + 4 * s2;
        const double ex = w[2] - w[0], ey = w[3] - w[1], den = dx * ey - dy * ex;
        if (fabs(den) < 1e-9) continue;
        const double t = ((w[0] - cx0) * ey - (w[1] - cy0) * ex) / den, u = ((w[0] - cx0) * dy - (w[1] - cy0) * dx) / den;
        f.through = u >= 0 && u <= 1 && t > 0 && (1 - t) * L > B.p.through_d;
      }
    }
    fs[k] = f;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  MapRec* R = &B.maps[m];
  const smg_params& P = B.p;
  long long st_obs = 0, st_floor = 0, st_ceil = 0, st_wall_tall = 0, st_through = 0, st_so_big = 0, st_wall = 0, st_wall_name = 0;
  int n_ceil = R->n_ceil;
  double ceil_est = R->ceil_est;
  int n = 0;
  for (int k = 0; k < nd; ++k) {
    const Fin& O = fs[k];
    if (!O.valid) {
      if (O.stage == 3) ++st_floor;
      continue;
    }
    if (O.through) { ++st_through; continue; }
    ++st_obs;
    bool drop = false;
    if (O.nc >= 8 && O.pl_ok && !(O.inl < P.plane_inl) && !(O.thick > P.plane_thick)) {
      const double nz = O.nz;
      if (nz > P.horiz) {
        if (O.zmed > 1.8) {
          if (n_ceil >= SMG_CEIL_OBS) {
            for (int i = 1; i < n_ceil; ++i) R->ceil_obs[i - 1] = R->ceil_obs[i];
            --n_ceil;
          }
          R->ceil_obs[n_ceil++] = O.zmed;
          if (n_ceil >= 20) {   // nth_element value at size/2
            const int kk = n_ceil / 2;
            double val = 0;
            for (int i = 0; i < n_ceil; ++i) {
              int less = 0, eq = 0;
              for (int j = 0; j < n_ceil; ++j) { less += R->ceil_obs[j] < R->ceil_obs[i]; eq += R->ceil_obs[j] == R->ceil_obs[i]; }
              if (less <= kk && kk < less + eq) { val = R->ceil_obs[i]; break; }
            }
            ceil_est = val;
          }
        }
        const double cz = ceil_est > 0 ? smin(P.ceil_z, ceil_est - P.ceil_band) : P.ceil_z;
        if (O.zmed > cz) { ++st_ceil; drop = true; }
        else if (O.zhi < P.floor_z) { ++st_floor; drop = true; }
      } else if (!(nz > P.wall_vert)) {
        // a thin upright plane that looks like structure: wall-like (objmap.cpp:594)
        if (O.ps >= 0.5) {
          B.obs[(size_t)m * B.max_det + k].wall_like = 1;
          B.obs[(size_t)m * B.max_det + k].struct_look = 1;
        }
        // named door / window / pillar / stairs within that shape's size (objmap.cpp:595-597)
        const int sh = O.so_sh;
        const bool so_keep = O.pso >= 0.5 && (sh == 1   ? O.hspan <= P.so_dw_w && O.zhi - O.zlo <= P.so_max_h
                                              : sh == 3 ? O.hspan <= P.so_pillar
                                                        : O.hspan <= P.so_stairs);
        const double cz = ceil_est > 0 ? ceil_est : P.ceil_z + 0.4;
        const bool tall = O.zhi - O.zlo >= P.tall_h || (O.zlo <= P.tall_floor && O.zhi >= cz - P.tall_ceil);
        const bool wide = O.hspan >= (O.ps >= P.tall_ps ? P.tall_w : P.tall_w_any);
        if (tall && wide && !so_keep) { ++st_wall_tall; drop = true; }
        else if (walls && !(O.w_near < P.wall_frac * O.w_tot) && !so_keep) {
          // a plane on a wall line (objmap.cpp:605-621): big -> wall, structure-named -> wall,
          // else kept as a wall-like fragment; a structural-object name keeps it within its size
          if (O.pso >= 0.5) ++st_so_big;
          if (smax(O.hspan, O.zhi - O.zlo) >= P.wall_big) { ++st_wall; drop = true; }
          else if (O.ps >= P.struct_p) { ++st_wall_name; drop = true; }
          else B.obs[(size_t)m * B.max_det + k].wall_like = 1;
        }
      }
    }
    if (!drop) B.obs_list[(size_t)m * B.max_det + n++] = k;
  }
  R->st.n_obs += st_obs;
  R->st.n_floor += st_floor;
  R->st.n_ceil += st_ceil;
  R->st.n_wall_tall += st_wall_tall;
  R->st.n_through += st_through;
  R->st.n_so_big += st_so_big;
  R->st.n_wall += st_wall;
  R->st.n_wall_name += st_wall_name;
  R->n_ceil = n_ceil;
  R->ceil_est = ceil_est;
  R->n_obs = n;
}
