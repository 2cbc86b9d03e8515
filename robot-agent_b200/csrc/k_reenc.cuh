// Whole-object re-encode requests of a keyframe (ObjectMap::buildReencode, scenemap
// src/objmap.cpp:1371-1458), run after the keyframe's cloud additions as the reference's push
// does (capi.cpp:1002-1010) on every frame that carries detection embeddings.
//
// For each confirmed object seen this keyframe with at least 30 cloud points, every stp-th cloud
// point (stp = max(1, n / 3000)) is projected into the frame.  A point in front of the depth
// surface (depth > 0 and depth >= z - 0.08) is visible: it paints a voxel-sized square
// (0.6 voxel at its depth) into the mask grid and its depth joins the median.  The painted mask
// is closed once (an empty cell with >= 3 painted neighbours of its 8 is filled), and the view
// kappa of the closed mask (sqrt(area) as size, median depth, visible fraction, truncation)
// decides the request.  Requests are ranked by priority (objects that never had a whole view
// first, then kappa over the best whole-view kappa) and the first reenc_max are kept.
//
// Layout: one CTA per (candidate slot, map).  Candidates are the objects that pass the cheap
// tests, numbered in list order; CTA x takes candidates x, x + gridDim.x, ...  The painted mask
// is a bitset in shared memory with rows padded to whole 32-bit words; the closing runs on
// whole words (the eight neighbour words are shifted copies of three rows, counted by a
// saturating bit-sliced adder) and writes the closed mask straight to the candidate's output
// slot, row-padded, so no second mask is held on chip.  Only the window of painted cells plus a
// one-cell ring is closed and written (no cell outside it has a painted neighbour); the window
// goes with the request and the reader zero-fills the rest.  The median depth is an exact radix
// selection over the visible depths kept in shared memory.  The last CTA of a map to finish
// ranks the candidates: priority descending, list order on equal priority (the reference's
// std::sort leaves the order of equal priorities unspecified).
#pragma once
#include "k_cloud.cuh"

#define RE_THREADS 256
#define RE_CTAS 16      // CTAs per map (a keyframe has about one candidate per detection)
#define RE_ZMAX 6000    // sampled points per object: ceil(n / max(1, n / 3000)) < 6000 for every n
// dynamic shared memory: the row-padded mask of the largest frame plus the visible depths
#define RE_SMEM(B) ((size_t)(B).H * ((((B).W) + 31) >> 5) * 4 + (size_t)RE_ZMAX * 4)

#define RE_PF 4        // points a thread projects at once (their loads in flight together)

// x / s with exact shortcuts: s == 1 (mode 0: x), s a power of two (mode 1: x * (1 / s), which
// rounds the same), otherwise a division (mode 2)
DEV int re_scale_mode(double s, double* inv) {
  int e;
  const double f = frexp(s, &e);
  *inv = 1.0 / s;
  return s == 1.0 ? 0 : (f == 0.5 ? 1 : 2);
}
DEV double re_scale(double x, double s, double inv, int mode) { return mode == 0 ? x : (mode == 1 ? x * inv : x / s); }

// order-preserving unsigned keys of floats
DEV uint32_t f_ord(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
DEV float f_unord(uint32_t k) { return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k); }

// k-th smallest (0-based, 0 <= k < n) of n floats: four most-significant-digit radix rounds of
// 8 bits; exact, so it is the value std::nth_element leaves at position k.
DEV float block_select_f(const float* a, int n, int k, int* hist, int* s_pick) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0, pmask = 0;
  for (int sh = 24; sh >= 0; sh -= 8) {
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int base = 0; base < n; base += blockDim.x) {   // one atomic per distinct bin of a warp
      const int i = base + tid;
      uint32_t key = 0;
      bool in = false;
      if (i < n) { key = f_ord(a[i]); in = (key & pmask) == prefix; }
      const uint32_t bin = (key >> sh) & 255u;
      const unsigned grp = __match_any_sync(0xffffffffu, in ? bin : 256u + (tid & 31));
      if (in && (tid & 31) == __ffs(grp) - 1) atomicAdd(&hist[bin], __popc(grp));
    }
    __syncthreads();
    if (tid < 32) {   // warp 0: the bin holding rank k (eight bins per lane)
      int c[8], sum = 0;
      for (int q = 0; q < 8; ++q) { c[q] = hist[tid * 8 + q]; sum += c[q]; }
      int incl = sum;
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += y;
      }
      int before = incl - sum;
      if (k >= before && k < incl) {
        int q = 0;
        while (q < 7 && k >= before + c[q]) { before += c[q]; ++q; }
        s_pick[0] = tid * 8 + q;
        s_pick[1] = k - before;
      }
    }
    __syncthreads();
    prefix |= (uint32_t)s_pick[0] << sh;
    pmask |= 255u << sh;
    k = s_pick[1];
    __syncthreads();
  }
  return f_unord(prefix);
}

// the cheap tests of objmap.cpp:1383 (every object here is an objprob object)
DEV bool reenc_candidate(const Batch& B, int m, const ObjRec& o, double stamp) {
  return o.confirmed && o.held_by < 0 && o.state != 1 && o.last_kf == stamp && B.clouds[cglob(B, m, o.cloud_slot)].n >= 30;
}

// viewKappa (bestview.cpp:77-81, objprob_math.h:78-87) with a visible fraction; the camera blur
// factor exp(-cam_w / blur_w) comes computed by the host libm
DEV double view_kappa_vis(const smg_params& P, double size_px, bool trunc, double depth, double vis, double blur_fac) {
  const double s = dmax2(0.0, size_px), d = dmax2(0.0, depth);
  double k = P.kap_k0 * s / (s + P.kap_s0);
  if (trunc) k *= P.kap_trunc;
  k /= 1.0 + (d / P.kap_d0) * (d / P.kap_d0);
  const double v = vis < 0 ? 0.0 : (vis > 1 ? 1.0 : vis);
  k *= P.kap_occ == 1.0 ? v : pow(v, P.kap_occ);
  if (P.kap_blur_w > 0) k *= blur_fac;
  return dmax2(k, 1e-3);
}

// Depth at pixel (u, v).  A device-resident frame is read directly.  For a host frame read in
// place (k_gather), the staging image holds the sample rows and each detection's scan box;
// any other pixel is read from the host frame.
DEV float reenc_depth(const FrameDev& F, int u, int v, int step, int stp, int& host_reads) {
  const size_t i = (size_t)v * F.w + u;
  if (!F.depth_host) return F.depth[i];
  if (v % step == 0 || (v >= stp / 2 && (v - stp / 2) % stp == 0)) return F.depth[i];
  for (int k = 0; k < F.n_det; ++k) {
    int u0, u1, v0, v1;
    det_scan_box(F, k, &u0, &u1, &v0, &v1);
    if (u >= u0 && u <= u1 && v >= v0 && v <= v1) return F.depth[i];
  }
  ++host_reads;
  return F.depth_host[i];
}

__global__ void __launch_bounds__(RE_THREADS) k_reenc(Batch B) {
  extern __shared__ __align__(16) unsigned char re_smem[];
  __shared__ BlockScratch bs;
  __shared__ int s_cand[RE_CAND];
  __shared__ int s_vis, s_last, s_nrec;
  __shared__ int s_hist[256], s_pick[2];
  const int m = B.map0 + blockIdx.y, tid = threadIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active) return;
  PHASE_START();
  MapRec* R = &B.maps[m];
  if (!(F.emb != nullptr && F.n_det > 0)) {   // not an objprob keyframe: no requests
    if (blockIdx.x == 0 && tid == 0) R->re_n = 0;
    return;
  }
  const smg_params& P = B.p;
  const double* T = F.T_mc;
  // the detector's mask grid and its affine to detector pixels; the label-image form has the
  // depth grid as its mask grid (scale 1, offset 0)
  const int mw = F.mask_w, mh = F.mask_h, img_w = F.img_w, img_h = F.img_h;
  const double msx = F.mask_sx, msy = F.mask_sy, mox = F.mask_ox, moy = F.mask_oy;
  const double sxu = F.sxu_d, syv = F.syv_d;
  double sxu_inv, syv_inv, msx_inv, msy_inv;
  const int sxu_mode = re_scale_mode(sxu, &sxu_inv), syv_mode = re_scale_mode(syv, &syv_inv);
  const int msx_mode = re_scale_mode(msx, &msx_inv), msy_mode = re_scale_mode(msy, &msy_inv);
  // footprint records of the candidate being projected: the CTA's cloud-add work area, free
  // once the keyframe's cloud additions are done (RE_CTAS <= WORK_SLOTS)
  uint2* recs_w = (uint2*)work_at(B, m, blockIdx.x).keys;
  const int wpr = (mw + 31) >> 5, nwords = mh * wpr;
  const int step = max(1, (int)llround(F.w / 160.0)), stp_mv = max(1, F.w / 32);
  uint32_t* g = (uint32_t*)re_smem;
  float* zs = (float*)(re_smem + (size_t)B.H * ((B.W + 31) >> 5) * 4);

  // candidates in list order; this CTA keeps its own
  const int nobj = R->n_obj;
  int ncand = 0;
  for (int b0 = 0; b0 < nobj; b0 += blockDim.x) {
    const int b = b0 + tid;
    int c = 0;
    if (b < nobj) c = reenc_candidate(B, m, B.objs[oglob(B, m, slot_at(B, m, b))], F.stamp);
    int tot;
    const int j = ncand + block_excl_scan(c, &tot, bs);
    if (c && j < RE_CAND && j % (int)gridDim.x == (int)blockIdx.x) s_cand[j / gridDim.x] = b;
    ncand += tot;
  }
  if (ncand > RE_CAND && blockIdx.x == 0 && tid == 0) set_err(R, SMG_E_CAP_REENC);
  const int nc = min(ncand, RE_CAND);
  __syncthreads();

  ReencRec* recs = B.reenc + (size_t)m * RE_CAND;
  int host_reads = 0;
  for (int i = tid; i < nwords; i += blockDim.x) g[i] = 0u;   // later candidates clear their window
  __syncthreads();
  PHASE_MARK(16);   // candidates + mask clear
  for (int q = 0; (int)blockIdx.x + q * (int)gridDim.x < nc; ++q) {
    const int j = blockIdx.x + q * gridDim.x;
    const int b = s_cand[q];
    const ObjRec& o = B.objs[oglob(B, m, slot_at(B, m, b))];
    const size_t cs = cglob(B, m, o.cloud_slot);
    const CloudRec& C = B.clouds[cs];
    const float4* pts = B.cpts + cs * B.cap;
    const int n = C.n;
    const int stp = max(1, n / 3000);
    const int tot = (n + stp - 1) / stp;
    if (tid == 0) { s_vis = 0; s_nrec = 0; }
    __syncthreads();
    double u0 = 1e9, v0 = 1e9, u1 = -1e9, v1 = -1e9;
    int trunc = 0;
    int pi0 = INT_MAX, pi1 = -1, pj0 = INT_MAX, pj1 = -1;   // painted cells of this thread
    // 1. projection and visibility: thread t takes points t, t + blockDim.x, ... (independent
    //    loads, RE_PF in flight per thread); a visible point appends its depth and, when its
    //    footprint meets the mask grid, the footprint's cell rectangle to the CTA's record list
    for (int base = 0; base < tot; base += RE_PF * (int)blockDim.x) {   // the same trip count for every thread
      float4 pt[RE_PF];
#pragma unroll
      for (int u = 0; u < RE_PF; ++u) {
        const int s = base + u * (int)blockDim.x + tid;
        pt[u] = s < tot && INB((size_t)s * stp, n, 801) ? pts[(size_t)s * stp] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      double czv[RE_PF], udv[RE_PF], vdv[RE_PF];
      float dv[RE_PF];
      bool in[RE_PF];
#pragma unroll
      for (int u = 0; u < RE_PF; ++u) {
        const int s = base + u * (int)blockDim.x + tid;
        const double p0 = C.org[0] + (double)pt[u].x - T[3], p1 = C.org[1] + (double)pt[u].y - T[7],
                     p2 = C.org[2] + (double)pt[u].z - T[11];
        const double cx = T[0] * p0 + T[4] * p1 + T[8] * p2, cy = T[1] * p0 + T[5] * p1 + T[9] * p2,
                     cz = T[2] * p0 + T[6] * p1 + T[10] * p2;
        czv[u] = cz;
        in[u] = s < tot && !(cz < 0.15);
        udv[u] = vdv[u] = 0;
        if (in[u]) {
          udv[u] = (double)F.fx * cx / cz + (double)F.cx;
          vdv[u] = (double)F.fy * cy / cz + (double)F.cy;
          if (udv[u] < 0 || vdv[u] < 0 || udv[u] >= F.w || vdv[u] >= F.h) { trunc = 1; in[u] = false; }
        }
      }
#pragma unroll
      for (int u = 0; u < RE_PF; ++u) dv[u] = in[u] ? reenc_depth(F, (int)udv[u], (int)vdv[u], step, stp_mv, host_reads) : 0.f;
#pragma unroll
      for (int u = 0; u < RE_PF; ++u) {
        const double cz = czv[u];
        const bool vis = in[u] && !(!(dv[u] > 0) || dv[u] < cz - 0.08);
        // depth pixel -> detector pixel -> mask cells over the voxel's footprint
        // (objmap.cpp:1403-1410; divisions by the scales, exact shortcuts for 1 and powers of 2)
        uint2 rec = make_uint2(0u, 0u);
        bool paint = false;
        if (vis) {
          const double ui = re_scale(udv[u], sxu, sxu_inv, sxu_mode), vi = re_scale(vdv[u], syv, syv_inv, syv_mode);
          const double rpx = re_scale(0.6 * P.voxel * (double)F.fx / cz, sxu, sxu_inv, sxu_mode);
          const int i0 = (int)floor(re_scale(ui - rpx - mox, msx, msx_inv, msx_mode));
          const int i1 = (int)floor(re_scale(ui + rpx - mox, msx, msx_inv, msx_mode));
          const int j0 = (int)floor(re_scale(vi - rpx - moy, msy, msy_inv, msy_mode));
          const int j1 = (int)floor(re_scale(vi + rpx - moy, msy, msy_inv, msy_mode));
          const int ia = max(0, i0), ib = min(mw - 1, i1), ja = max(0, j0), jb = min(mh - 1, j1);
          if (ia <= ib && ja <= jb) {
            pi0 = min(pi0, ia); pi1 = max(pi1, ib); pj0 = min(pj0, ja); pj1 = max(pj1, jb);
            rec = make_uint2((uint32_t)ia | (uint32_t)ib << 16, (uint32_t)ja | (uint32_t)jb << 16);
            paint = true;
          }
          u0 = fmin(u0, ui); u1 = fmax(u1, ui); v0 = fmin(v0, vi); v1 = fmax(v1, vi);
          if (ui <= 2 || vi <= 2 || ui >= img_w - 3 || vi >= img_h - 3) trunc = 1;
        }
        // append the depth and the footprint: one shared-memory atomic per warp each
        const unsigned bv = __ballot_sync(0xffffffffu, vis), bp = __ballot_sync(0xffffffffu, paint);
        const int lane = tid & 31;
        int zb = 0, rb = 0;
        if (lane == 0) {
          if (bv) zb = atomicAdd(&s_vis, __popc(bv));
          if (bp) rb = atomicAdd(&s_nrec, __popc(bp));
        }
        zb = __shfl_sync(0xffffffffu, zb, 0);
        rb = __shfl_sync(0xffffffffu, rb, 0);
        if (vis) {
          const int zi = zb + __popc(bv & ((1u << lane) - 1u));
          if (INB(zi, RE_ZMAX, 802)) zs[zi] = (float)cz;
        }
        if (paint) {
          const int ri = rb + __popc(bp & ((1u << lane) - 1u));
          if (INB(ri, RE_ZMAX, 804)) recs_w[ri] = rec;
        }
      }
    }
    __syncthreads();
    // 2. paint the footprints: thread t takes a run of consecutive records (points that are
    //    neighbours in the cloud paint the same words, which the thread then finds painted, and
    //    the lanes of a warp work on distant parts instead of contending for one word)
    {
      const int nrec = min(s_nrec, RE_ZMAX);
      const int per = (nrec + (int)blockDim.x - 1) / (int)blockDim.x;
      for (int r = tid * per, r_end = min(nrec, r + per); r < r_end; ++r) {
        const uint2 rec = recs_w[r];
        const int ia = (int)(rec.x & 0xffffu), ib = (int)(rec.x >> 16), ja = (int)(rec.y & 0xffffu), jb = (int)(rec.y >> 16);
        for (int jj = ja; jj <= jb; ++jj) {
          uint32_t* row = g + (size_t)jj * wpr;
          for (int u = ia; u <= ib;) {
            const int w = u >> 5, e = min(ib, (w << 5) + 31);
            const uint32_t bits = (e - u == 31) ? 0xffffffffu : (((1u << (e - u + 1)) - 1u) << (u & 31));
            if ((row[w] & bits) != bits) atomicOr(&row[w], bits);
            u = e + 1;
          }
        }
      }
    }
    trunc = __syncthreads_or(trunc);
    PHASE_MARK(17);   // projection + paint
    const int vis = s_vis;
    u0 = block_min_d(u0, bs); u1 = block_max_d(u1, bs);
    v0 = block_min_d(v0, bs); v1 = block_max_d(v1, bs);
    // window of the closing: painted cells plus a one-cell ring, in whole words
    pi0 = (int)block_min_d((double)pi0, bs); pi1 = (int)block_max_d((double)pi1, bs);
    pj0 = (int)block_min_d((double)pj0, bs); pj1 = (int)block_max_d((double)pj1, bs);
    const bool painted = pi1 >= 0;
    const int r0 = painted ? max(0, pj0 - 1) : 0, r1 = painted ? min(mh - 1, pj1 + 1) : -1;
    const int w0 = painted ? max(0, pi0 - 1) >> 5 : 0, w1 = painted ? min(mw - 1, pi1 + 1) >> 5 : -1;
    const int nww = w1 - w0 + 1, nwin = painted ? (r1 - r0 + 1) * nww : 0;
    bool ok = tot > 0 && vis >= 12;
    const double vfrac = ok ? (double)vis / tot : 0.0;
    ok = ok && !(vfrac < P.reenc_min_vis);
    double size_px = 0;
    if (ok) {   // closing by one cell, written to the candidate's output slot; area of the result
      uint32_t* out = B.reenc_bits + ((size_t)m * RE_CAND + j) * B.re_words;
      const uint32_t tail = (mw & 31) ? (1u << (mw & 31)) - 1u : 0xffffffffu;
      long long area = 0;
      for (int t = tid; t < nwin; t += blockDim.x) {
        const int r = r0 + t / nww, w = w0 + t % nww;
        uint32_t s0 = 0, s1 = 0, s2 = 0;
        auto add = [&](uint32_t x) { const uint32_t c0 = s0 & x; s0 ^= x; const uint32_t c1 = s1 & c0; s1 ^= c0; s2 |= c1; };
        for (int dr = -1; dr <= 1; ++dr) {
          const int rr = r + dr;
          if (rr < 0 || rr >= mh) continue;
          const uint32_t* row = g + (size_t)rr * wpr;
          const uint32_t c = row[w], l = w > 0 ? row[w - 1] : 0u, h = w + 1 < wpr ? row[w + 1] : 0u;
          add((c << 1) | (l >> 31));   // left neighbour (column - 1)
          add((c >> 1) | (h << 31));   // right neighbour (column + 1)
          if (dr != 0) add(c);
        }
        uint32_t g2 = g[(size_t)r * wpr + w] | s2 | (s1 & s0);   // painted, or >= 3 painted neighbours
        if (w == wpr - 1) g2 &= tail;
        out[(size_t)r * wpr + w] = g2;
        area += __popc(g2);
      }
      area = block_sum_ll(area, bs);
      size_px = sqrt((double)area * msx * msy);
      ok = !(size_px < (double)P.reenc_min_px);
    }
    PHASE_MARK(18);   // windows + closing
    float zmed = 0.f;
    if (ok) zmed = block_select_f(zs, min(vis, RE_ZMAX), vis / 2, s_hist, s_pick);
    PHASE_MARK(19);   // median
    if (tid == 0) {
      ReencRec rc;
      rc.id = o.id;
      rc.ok = 0;
      rc.prio = 0;
      rc.kappa = 0.f;
      rc.mask_w = mw;
      rc.mask_h = mh;
      rc.win[0] = r0; rc.win[1] = r1; rc.win[2] = w0; rc.win[3] = w1;
      if (ok) {
        // ViewQuality holds float fields (bestview.hpp:58-64)
        const float size_f = (float)size_px, vis_f = (float)vfrac;
        const double kap = view_kappa_vis(P, (double)fmaxf(0.f, size_f), trunc != 0, (double)fmaxf(0.f, zmed), (double)vis_f, F.blur_fac);
        const bool need = o.need_whole != 0;
        if (need || !(kap < P.reenc_gain * o.whole_kappa)) {
          rc.ok = 1;
          rc.prio = (need ? 1e6 : 0.0) + kap / dmax2(1.0, o.whole_kappa);
          rc.kappa = (float)kap;
          rc.box[0] = (float)dmax2(0.0, u0 - 2);
          rc.box[1] = (float)dmax2(0.0, v0 - 2);
          rc.box[2] = (float)dmin2((double)img_w, u1 + 2);
          rc.box[3] = (float)dmin2((double)img_h, v1 + 2);
          for (int k = 0; k < 6; ++k) rc.cam[k] = k < 3 ? T[4 * k + 3] : T[4 * (k - 3) + 2];
        }
      }
      recs[j] = rc;
    }
    for (int t = tid; t < nwin; t += blockDim.x) g[(size_t)(r0 + t / nww) * wpr + w0 + t % nww] = 0u;   // painted cells lie inside
    __syncthreads();
  }
  PHASE_MARK(20);   // records + window clears
  host_reads = __reduce_add_sync(0xffffffffu, host_reads);
  if ((tid & 31) == 0 && host_reads) wk_add(R, SMG_WK_H2D, 4LL * host_reads);

  // the last CTA of the map ranks the candidates
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(&R->re_done, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  int n_ok = 0;
  for (int j = tid; j < nc; j += blockDim.x) {
    if (!__ldcg(&recs[j].ok)) continue;
    ++n_ok;
    const double pj = __ldcg(&recs[j].prio);
    int rank = 0;
    for (int k = 0; k < nc; ++k) {
      if (k == j || !__ldcg(&recs[k].ok)) continue;
      const double pk = __ldcg(&recs[k].prio);
      rank += pk > pj || (pk == pj && k < j);
    }
    if (rank < P.reenc_max && INB(rank, RE_CAND, 803)) R->re_rank[rank] = j;
  }
  n_ok = block_sum_i(n_ok, bs);
  PHASE_MARK(21);   // ranking (last CTA)
  if (tid == 0) {
    const int nreq = min(n_ok, max(0, P.reenc_max));
    R->re_n = nreq;
    R->st.n_reenc_req += nreq;
    R->re_done = 0;
  }
}
