// Standalone 2D occupancy + correlative scan matching.
//
// OccGrid::insert (scenemap src/grid.cpp:95-159, hit/miss :57-93) for M independent grids,
// spread over many CTAs per grid: a first pass takes, per cell, the minimum of a first-touch
// key (scan id in the high word, then hits in point order before every ray cell, rays in
// order, cells along a ray in step order) with atomicMin; the second pass lets only the
// occurrence holding a cell's key apply its update.  That is exactly the reference's "one
// update per cell per scan, hits first, first writer wins" with a sequential loop.
//
// Correlative scan matching (real-time correlative search as configured for the reference's
// Cartographer front end, slam_carto/config/carto_2d.lua:17-21): candidate poses are 2K+1
// rotations of the hit points about the initial pose, each discretised to cells once, plus
// integer cell offsets in x and y.  A candidate's score is the sum over the points of the
// cell's occupancy probability quantised to uint16 (OccGrid::prob, grid.cpp:261-266: unseen
// or outside = pmin), i.e. an integer, then normalised by the point count and weighted by
// exp(-(|t| w_t + |dth| w_r)^2) with host-libm weights.  The best candidate is the maximum,
// the lowest candidate index (rotation, then x offset, then y offset) on ties.
#pragma once
#include "dev_util.cuh"

#define OCC_THREADS 256
#define CSM_SECTORS 8
#define CSM_MAX_ROT 81
#define CSM_MAX_LIN 13
#define CSM_WIN_CELLS 49152   // shared-memory window (uint16) per CTA; larger windows read L2

struct OccDev {
  int M, W, H, X0, Y0;   // grid window in global cell indices
  float res;
  int q_hit, q_miss, q_min, q_max, lut_off;
  uint16_t q_unseen;
  int16_t* L;
  int8_t* c8;
  uint8_t* flags;        // 1 = seen, 2 = point sums valid
  float4* cold;          // sx, sy, nx, ny
  uint32_t* cnt;         // cnt | cntn << 16
  unsigned long long* touch;
  uint16_t* Q;           // quantised occupancy probability (the matcher's grid)
  const int8_t* lut8;
  const uint16_t* qlut;
  uint32_t* scan_id;     // [M]
  int32_t* changed;      // [M]
  int32_t* err;          // [M] 1 = point outside the window
  // per-call scan inputs (device copies)
  int max_pts;
  float2* pts;           // [M][3*max_pts]: match points, laser hits, free ends (base frame)
  float2* mn;            // [M][max_pts] match-point normals
  int32_t* nmhf;         // [M][3] counts: match, hit, free
  float2* origin;        // [M] sensor origin, base frame
  double* pose;          // [M][5]: x, y, th, cos th, sin th of the insert pose
  // matcher
  int n_rot, n_lin, lin_half;
  double* rot;           // [M][n_rot][2] cos, sin of th0 + (j - half) * step
  double* pose0;         // [M][3]
  const double* cand_w;  // [n_rot * n_lin * n_lin]
  double lin_step;       // metres per cell offset (= res)
  double ang_step;
  uint32_t* score;       // [M][n_rot * n_lin * n_lin]
  int32_t* best;         // [M]
  double* best_score;    // [M]
};

DEV int occ_cell(double v, float res) { return (int)floor(v / (double)res); }

DEV uint16_t occ_q(const OccDev& G, int m, int ix, int iy) {
  if (ix < G.X0 || iy < G.Y0 || ix >= G.X0 + G.W || iy >= G.Y0 + G.H) return G.q_unseen;
  return G.Q[(size_t)m * G.W * G.H + (size_t)(iy - G.Y0) * G.W + (ix - G.X0)];
}

// ---------------------------------------------------------------- matcher
// grid (CSM_SECTORS, n_rot, M): the hit points of sector s, rotated by candidate rotation j,
// scored against every (x, y) offset; integer partial sums go to score[m][j][*] atomically.
__global__ void __launch_bounds__(OCC_THREADS) k_csm_score(OccDev G) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint16_t* win = (uint16_t*)smem_raw;
  __shared__ int cx_[1024], cy_[1024];
  __shared__ BlockScratch bs;
  const int s = blockIdx.x, j = blockIdx.y, m = blockIdx.z, tid = threadIdx.x;
  const int nhit = G.nmhf[3 * m + 1], nm = G.nmhf[3 * m];
  const int p0 = (int)((long long)s * nhit / gridDim.x), p1 = (int)((long long)(s + 1) * nhit / gridDim.x);
  const int np = p1 - p0;
  if (np <= 0 || np > 1024) return;
  const double* P = G.pose0 + 3 * m;
  const double c = G.rot[((size_t)m * G.n_rot + j) * 2], sn = G.rot[((size_t)m * G.n_rot + j) * 2 + 1];
  const float2* hp = G.pts + (size_t)m * 3 * G.max_pts + nm + p0;
  int lx = 1 << 30, ly = 1 << 30, hx = -(1 << 30), hy = -(1 << 30);
  for (int i = tid; i < np; i += blockDim.x) {
    const float2 q = hp[i];
    const double wx = P[0] + c * (double)q.x - sn * (double)q.y, wy = P[1] + sn * (double)q.x + c * (double)q.y;
    const int ix = occ_cell(wx, G.res), iy = occ_cell(wy, G.res);
    cx_[i] = ix;
    cy_[i] = iy;
    lx = min(lx, ix); ly = min(ly, iy); hx = max(hx, ix); hy = max(hy, iy);
  }
  const int H2 = G.lin_half;
  const int bx0 = (int)block_min_d((double)lx, bs) - H2, by0 = (int)block_min_d((double)ly, bs) - H2;
  const int bx1 = (int)block_max_d((double)hx, bs) + H2, by1 = (int)block_max_d((double)hy, bs) + H2;
  const int ww = bx1 - bx0 + 1, wh = by1 - by0 + 1;
  const bool staged = (long long)ww * wh <= CSM_WIN_CELLS;
  if (staged) {
    for (int k = tid; k < ww * wh; k += blockDim.x) {
      const int yy = k / ww, xx = k - yy * ww;
      win[k] = occ_q(G, m, bx0 + xx, by0 + yy);
    }
  }
  __syncthreads();
  const int nl = G.n_lin, nt = nl * nl;
  uint32_t* S = G.score + ((size_t)m * G.n_rot + j) * nt;
  // thread t = x offset * n_lin + y offset (candidate order inside a rotation)
  for (int t = tid; t < nt; t += blockDim.x) {
    const int kx = t / nl - H2, ky = t % nl - H2;
    uint32_t sum = 0;
    if (staged) {
      for (int i = 0; i < np; ++i) sum += win[(cy_[i] + ky - by0) * ww + (cx_[i] + kx - bx0)];
    } else {
      for (int i = 0; i < np; ++i) sum += occ_q(G, m, cx_[i] + kx, cy_[i] + ky);
    }
    atomicAdd(&S[t], sum);
  }
}

// one CTA per grid: best candidate (max weighted score, lowest index on ties), the insert pose
// it implies, and the score counters cleared for the next call
__global__ void __launch_bounds__(OCC_THREADS) k_csm_best(OccDev G) {
  __shared__ double wb[OCC_THREADS / 32];
  __shared__ int wi[OCC_THREADS / 32];
  const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int nl = G.n_lin, nc = G.n_rot * nl * nl;
  const int nhit = G.nmhf[3 * m + 1];
  uint32_t* S = G.score + (size_t)m * nc;
  const double den = (double)nhit * 65535.0;
  double bv = -1.0;
  int bi = 0x7fffffff;
  for (int k = tid; k < nc; k += blockDim.x) {
    const double v = nhit > 0 ? ((double)S[k] / den) * G.cand_w[k] : 0.0;
    if (v > bv || (v == bv && k < bi)) { bv = v; bi = k; }
    S[k] = 0;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const double v2 = __shfl_xor_sync(0xffffffffu, bv, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    if (v2 > bv || (v2 == bv && i2 < bi)) { bv = v2; bi = i2; }
  }
  if (lane == 0) { wb[wid] = bv; wi[wid] = bi; }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (wb[w] > bv || (wb[w] == bv && wi[w] < bi)) { bv = wb[w]; bi = wi[w]; }
    if (nhit <= 0) { bi = ((G.n_rot / 2) * nl + G.lin_half) * nl + G.lin_half; bv = 0.0; }
    const int j = bi / (nl * nl), r = bi - j * nl * nl, kx = r / nl - G.lin_half, ky = r % nl - G.lin_half;
    const double* P = G.pose0 + 3 * m;
    double* Q = G.pose + 5 * m;
    Q[0] = P[0] + (double)kx * G.lin_step;
    Q[1] = P[1] + (double)ky * G.lin_step;
    Q[2] = P[2] + (double)(j - G.n_rot / 2) * G.ang_step;
    Q[3] = G.rot[((size_t)m * G.n_rot + j) * 2];
    Q[4] = G.rot[((size_t)m * G.n_rot + j) * 2 + 1];
    G.best[m] = bi;
    G.best_score[m] = bv;
  }
}

// ---------------------------------------------------------------- insert
// item k of map m: k < nm match point, < nm+nh laser hit, else free-ray end (grid.cpp:207-214)
DEV void occ_item(const OccDev& G, int m, int k, double* wx, double* wy) {
  const double* Q = G.pose + 5 * m;
  const float2 p = G.pts[(size_t)m * 3 * G.max_pts + k];
  *wx = Q[0] + Q[3] * (double)p.x - Q[4] * (double)p.y;
  *wy = Q[1] + Q[4] * (double)p.x + Q[3] * (double)p.y;
}

DEV bool occ_inside(const OccDev& G, int ix, int iy) {
  return ix >= G.X0 && iy >= G.Y0 && ix < G.X0 + G.W && iy < G.Y0 + G.H;
}

// Bresenham walk of ray r (grid.cpp:236-256) from the origin cell; visit(ci, step) per cell,
// the end cell included only for free rays
template <class F>
DEV void occ_ray(const OccDev& G, int cx, int cy, int x1, int y1, bool end_incl, F visit) {
  int x = cx, y = cy;
  const int dx = abs(x1 - x), dy = -abs(y1 - y), sx = x < x1 ? 1 : -1, sy = y < y1 ? 1 : -1;
  int err = dx + dy;
  unsigned step = 0;
  for (;;) {
    const bool end = x == x1 && y == y1;
    if (end && !end_incl) break;
    visit((size_t)(y - G.Y0) * G.W + (x - G.X0), step);
    if (end) break;
    ++step;
    const int e2 = 2 * err;
    if (e2 >= dy) { err += dy; x += sx; }
    if (e2 <= dx) { err += dx; y += sy; }
  }
}

DEV void occ_origin(const OccDev& G, int m, int* cx, int* cy) {
  const double* Q = G.pose + 5 * m;
  const float2 o = G.origin[m];
  const double ox = Q[0] + Q[3] * (double)o.x - Q[4] * (double)o.y, oy = Q[1] + Q[4] * (double)o.x + Q[3] * (double)o.y;
  *cx = occ_cell(ox, G.res);
  *cy = occ_cell(oy, G.res);
}

// The scan id is advanced by the host-side launch sequence (k_occ_begin), so every CTA of the
// touch and apply passes reads the same value.
__global__ void k_occ_begin(OccDev G) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= G.M) return;
  ++G.scan_id[m];
  G.changed[m] = 0;
  G.err[m] = 0;
}

// pass 1 (grid (blocks, M)): bounds check, then first-touch keys of every hit and ray cell
__global__ void __launch_bounds__(OCC_THREADS) k_occ_keys(OccDev G) {
  const int m = blockIdx.y;
  const int nm = G.nmhf[3 * m], nh = G.nmhf[3 * m + 1], nf = G.nmhf[3 * m + 2], n = nm + nh + nf;
  const unsigned long long sk = (unsigned long long)(0xffffffffu - G.scan_id[m]) << 32;
  unsigned long long* T = G.touch + (size_t)m * G.W * G.H;
  int cx, cy;
  occ_origin(G, m, &cx, &cy);
  if (!occ_inside(G, cx, cy)) {
    if (threadIdx.x == 0) G.err[m] = 1;
    return;
  }
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < n; k += gridDim.x * blockDim.x) {
    double wx, wy;
    occ_item(G, m, k, &wx, &wy);
    const int ix = occ_cell(wx, G.res), iy = occ_cell(wy, G.res);
    if (!occ_inside(G, ix, iy)) { G.err[m] = 1; continue; }
    if (k < nm + nh) atomicMin(&T[(size_t)(iy - G.Y0) * G.W + (ix - G.X0)], sk | (unsigned)k);
    if (k >= nm) {
      const unsigned r = (unsigned)(k - nm);
      occ_ray(G, cx, cy, ix, iy, k >= nm + nh, [&](size_t ci, unsigned step) {
        atomicMin(&T[ci], sk | 0x80000000ull | ((unsigned long long)r << 12) | (step & 0xfffu));
      });
    }
  }
}

// pass 2: the occurrence that holds a cell's key applies hit (grid.cpp:157-173) or miss
// (grid.cpp:175-193); the quantised probability follows every applied update
__global__ void __launch_bounds__(OCC_THREADS) k_occ_apply(OccDev G) {
  __shared__ int sh_ch;
  const int m = blockIdx.y;
  if (G.err[m]) return;
  if (threadIdx.x == 0) sh_ch = 0;
  __syncthreads();
  const int nm = G.nmhf[3 * m], nh = G.nmhf[3 * m + 1], nf = G.nmhf[3 * m + 2], n = nm + nh + nf;
  const unsigned long long sk = (unsigned long long)(0xffffffffu - G.scan_id[m]) << 32;
  const size_t base = (size_t)m * G.W * G.H;
  const unsigned long long* T = G.touch + base;
  const double* Q = G.pose + 5 * m;
  int cx, cy;
  occ_origin(G, m, &cx, &cy);
  int ch = 0;
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < n; k += gridDim.x * blockDim.x) {
    double wx, wy;
    occ_item(G, m, k, &wx, &wy);
    const int ix = occ_cell(wx, G.res), iy = occ_cell(wy, G.res);
    const size_t ci = (size_t)(iy - G.Y0) * G.W + (ix - G.X0);
    if (k < nm + nh && T[ci] == (sk | (unsigned)k)) {
      float nx = 0.f, ny = 0.f;
      if (k < nm) {
        const float2 q = G.mn[(size_t)m * G.max_pts + k];
        nx = (float)(Q[3] * (double)q.x - Q[4] * (double)q.y);
        ny = (float)(Q[4] * (double)q.x + Q[3] * (double)q.y);
      }
      const size_t g = base + ci;
      const int L = G.L[g];
      const int nL = min(L + G.q_hit, G.q_max);
      const bool was_seen = G.flags[g] & 1;
      G.flags[g] |= 3;
      ch += (nL != L) | !was_seen;
      G.L[g] = (int16_t)nL;
      G.c8[g] = G.lut8[nL + G.lut_off];
      G.Q[g] = G.qlut[nL + G.lut_off];
      float4 cs = G.cold[g];
      uint32_t cnt = G.cnt[g];
      uint32_t c1 = cnt & 0xffffu, c2 = cnt >> 16;
      if (c1 < 60000) { cs.x += (float)wx; cs.y += (float)wy; ++c1; }
      if ((nx != 0 || ny != 0) && c2 < 60000) { cs.z += nx; cs.w += ny; ++c2; }
      G.cold[g] = cs;
      G.cnt[g] = c1 | c2 << 16;
    }
    if (k >= nm) {
      const unsigned r = (unsigned)(k - nm);
      occ_ray(G, cx, cy, ix, iy, k >= nm + nh, [&](size_t cj, unsigned step) {
        if (T[cj] != (sk | 0x80000000ull | ((unsigned long long)r << 12) | (step & 0xfffu))) return;
        const size_t g = base + cj;
        const int L = G.L[g];
        const int nL = max(L + G.q_miss, G.q_min);
        const bool was_seen = G.flags[g] & 1;
        G.flags[g] |= 1;
        if (nL == L && was_seen) return;
        ++ch;
        G.L[g] = (int16_t)nL;
        G.c8[g] = G.lut8[nL + G.lut_off];
        G.Q[g] = G.qlut[nL + G.lut_off];
        if (nL <= 0 && (G.flags[g] & 2)) {
          G.flags[g] &= (uint8_t)~2u;
          G.cold[g] = make_float4(0.f, 0.f, 0.f, 0.f);
          G.cnt[g] = 0;
        }
      });
    }
  }
  if (ch) atomicAdd(&sh_ch, ch);
  __syncthreads();
  if (threadIdx.x == 0 && sh_ch) atomicAdd(&G.changed[m], sh_ch);
}
