// Wall segments from each map's own occupancy grid, before the object update of the keyframe,
// as the reference's image push runs them (scenemap capi.cpp:646-698 refreshWalls, :866-890 the
// bridged list handed to ObjectMap::update as ObjFrame::wall_segs; walls.cpp: wallSegments /
// WallExtractor::update, wallAngle, wallSegmentsAtAngle; walls.hpp constants).
//
//  - k_wall_rects (object stream, before the hands step): the floor footprints of confirmed,
//    exportable objects that wall extraction ignores (capi.cpp:649-658), in object order, and
//    whether they differ from the set of the last extraction.
//  - k_walls (grid stream, after k_grid): the refresh policy (dominant-direction re-measure every
//    2 s of stamps when the grid or the footprints changed, 1-degree hysteresis; axis-aligned maps
//    re-extract on every change, tilted ones at most every 0.5 s), the extraction itself, and the
//    keyframe's list: the extracted segments plus the window bridges between collinear ones.
//    One CTA per map.  The occupancy of the window becomes row bits (top row first) and, by
//    warp ballots, column bits; runs of occupied cells along rows and along columns are found
//    word-wise in parallel (a thread per row / column), and one warp per direction chains runs of consecutive rows (columns) into groups
//    in the reference's order (a ballot picks the first open group a run overlaps), emitting
//    each group's centre line.
//    The dominant direction scores all candidate angles of a stage at once: each group of
//    threads fills its own shared-memory projection histograms.
//  - k_wall_state: sm_snap_wall_state (capi.cpp:1239-1245, walls.cpp rayDistances /
//    segmentsRobotFrame / wallStateVector) for one map and pose.
// Cells are the library's grid window: the reference computes the same functions on its own
// grown grid, whose extent only shifts the direction histograms' bin phase and the cell
// rounding of the ignore rectangles.
#pragma once
#include "dev_util.cuh"

#define WALL_THREADS 1024
#define WALL_SMEM (96 * 1024)
#define WALL_OCC 65                   // kOccMin (walls.hpp:15)
#define WALL_MIN_LEN 0.5              // kMinLen
#define WALL_MAX_THICK 0.5            // kMaxThick
#define WALL_OVERLAP 0.6              // the overlap refreshWalls passes
#define WALL_PI 3.14159265358979323846
#define WALL_ALIGN_TOL (1.0 * WALL_PI / 180.0)   // kAlignTol
#define WALL_ALIGN_GAIN 1.08          // kAlignGain
#define WALL_ANGLE_EVERY 2.0          // kWallAngleEvery (capi.cpp:88)
#define WALL_ANGLE_HYST (WALL_PI / 180.0)        // kWallAngleHyst
#define WALL_ALIGNED_EVERY 0.5        // kWallAlignedEvery
#define WALL_ACT_MAX 1024             // open groups of one row (runs per row)
#define WALL_SECTORS 16               // kSectors
#define WALL_SEGMENTS 8               // kSegments
#define WALL_MAX_RANGE 4.0            // kMaxRange
#define WALL_STATE_LEN (WALL_SECTORS + WALL_SEGMENTS * 5)

// ---- the ignore footprints ----------------------------------------------------------------

// Objects whose floor footprint wall extraction ignores (capi.cpp:649-658): exportable
// (confirmed, named, not hidden, not the fallback name, not a structure label), not held, not
// gone, reaching down to 0.4 m, not wall-like, not a structural object, at most 5 m wide.
DEV bool wall_ignores(const Batch& B, const ObjRec& o) {
  if (!exportable(B, o) || kind_of(B, o.cls) == KIND_STRUCT_OBJ) return false;
  if (o.held_by >= 0 || o.state == 1 || o.lo[2] > 0.4 || o.wall_like) return false;
  const double dx = o.hi[0] - o.lo[0], dy = o.hi[1] - o.lo[1];
  return !(dx > 5.0 || dy > 5.0);
}

__global__ void __launch_bounds__(256) k_wall_rects(Batch B) {
  __shared__ int scan_db[2][33];
  __shared__ BlockScratch bs;
  const int m = B.map0 + blockIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active || !B.walls_on) return;
  MapRec* R = &B.maps[m];
  const int n = R->n_obj;
  double* rect = B.wrect + (size_t)m * B.O * 4;
  int before = 0, it = 0;
  for (int c0 = 0; c0 < n; c0 += blockDim.x) {
    const int b = c0 + threadIdx.x;
    int need = 0;
    const ObjRec* o = nullptr;
    if (b < n) {
      o = &B.objs[oglob(B, m, slot_at(B, m, b))];
      need = wall_ignores(B, *o);
    }
    int tot;
    const int r = before + block_scan_db(need, &tot, scan_db, it++);
    if (need && INB(r, B.O, 1101)) {
      rect[4 * r] = o->lo[0] - 0.1;
      rect[4 * r + 1] = o->lo[1] - 0.1;
      rect[4 * r + 2] = o->hi[0] + 0.1;
      rect[4 * r + 3] = o->hi[1] + 0.1;
    }
    before += tot;
  }
  __syncthreads();
  const int nr = min(before, B.O);
  const double* prev = B.wrect_prev + (size_t)m * B.O * 4;
  int diff = 0;
  if (nr == R->n_rect_prev)
    for (int i = threadIdx.x; i < 4 * nr; i += blockDim.x) diff += rect[i] != prev[i];
  diff = block_sum_i(diff, bs);
  if (threadIdx.x == 0) {
    R->n_rect = nr;
    R->w_rchg = nr != R->n_rect_prev || diff != 0;
  }
}

// ---- extraction ---------------------------------------------------------------------------

// Occupancy bits of a w x h grid, top row first (bit row iy = grid row h - 1 - iy, as the
// reference's PGM row order): cell set when >= kOccMin and outside every ignore rectangle (cell
// ranges x0..x1, y0..y1 inclusive, in grid rows).
DEV void wall_bits(const int8_t* cells, int w, int h, int nw, uint64_t* bits, const int4* rc0, const int4* rc1, int n_rc) {
  for (int i = threadIdx.x; i < h * nw; i += blockDim.x) {
    const int iy = i / nw, k = i - iy * nw, y = h - 1 - iy;
    const int8_t* row = cells + (size_t)y * w;
    const int x0 = k * 64, x1 = min(w, x0 + 64);
    uint64_t v = 0;
    if (x1 - x0 == 64 && (((size_t)(row + x0)) & 15) == 0) {   // four 16-byte loads in flight
      uint4 q[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) q[j] = ((const uint4*)(row + x0))[j];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t wd[4] = {q[j].x, q[j].y, q[j].z, q[j].w};
#pragma unroll
        for (int e = 0; e < 16; ++e) v |= (uint64_t)((int8_t)(wd[e >> 2] >> (8 * (e & 3))) >= WALL_OCC) << (16 * j + e);
      }
    } else {
      for (int x = x0; x < x1; ++x) v |= (uint64_t)(row[x] >= WALL_OCC) << (x - x0);
    }
    for (int r = 0; r < n_rc && v; ++r) {
      const int4 a = rc0[r], b = rc1[r];   // a = (x0, y0), b = (x1, y1)
      if (y < a.y || y > b.y || b.x < x0 || a.x >= x1) continue;
      const int lo = max(a.x, x0) - x0, hi = min(b.x, x1 - 1) - x0;
      const uint64_t msk = hi - lo == 63 ? ~0ull : (((1ull << (hi - lo + 1)) - 1ull) << lo);
      v &= ~msk;
    }
    bits[i] = v;
  }
}

// Runs of set bits of every row with at least min_run cells (a thread per row): run = a | b << 16.
DEV void wall_row_runs(const uint64_t* bits, int h, int nw, int min_run, uint32_t* runs, int rp, int32_t* cnt, int* ovf) {
  for (int iy = threadIdx.x; iy < h; iy += blockDim.x) {
    const uint64_t* row = bits + (size_t)iy * nw;
    int n = 0, open = -1;
    uint64_t carry = 0;
    for (int k = 0; k < nw; ++k) {
      const uint64_t v = row[k];
      uint64_t t = v ^ ((v << 1) | carry);   // bit p: cell p differs from cell p - 1
      carry = v >> 63;
      while (t) {
        const int p = k * 64 + __ffsll((long long)t) - 1;
        t &= t - 1;
        if (open < 0) {
          open = p;
        } else {
          if (p - open >= min_run) {
            if (n < rp) runs[(size_t)iy * rp + n] = (uint32_t)open | (uint32_t)(p - 1) << 16;
            ++n;
          }
          open = -1;
        }
      }
    }
    if (open >= 0 && nw * 64 - open >= min_run) {
      if (n < rp) runs[(size_t)iy * rp + n] = (uint32_t)open | (uint32_t)(nw * 64 - 1) << 16;
      ++n;
    }
    if (n > rp) atomicOr(ovf, 1);
    cnt[iy] = min(n, rp);
  }
}

struct WallOut {
  double* seg;   // n x 4
  int cap, n, ovf;
};

// A group's centre line (walls.cpp update's emit): groups thicker than max_thick are skipped;
// transposed groups come from column runs.
DEV void wall_emit(const int4& g, bool transpose, int h, double res, double ox, double oy, WallOut& o) {
  if ((g.y - g.x + 1) * res > WALL_MAX_THICK) return;   // (r1 - r0 + 1) * res
  const double rc = (g.x + g.y) / 2.0;
  if (o.n >= o.cap) { o.ovf = 1; return; }
  double* s = o.seg + 4 * (size_t)o.n++;
  for (int e = 0; e < 2; ++e) {
    const int c = e ? g.w : g.z;
    const double iy = transpose ? (double)c : rc, ix = transpose ? rc : (double)c;
    s[2 * e] = ox + (ix + 0.5) * res;
    s[2 * e + 1] = oy + ((double)(h - 1) - iy + 0.5) * res;
  }
}

// groupRuns by one warp: the runs of consecutive rows chain into groups; a run joins the first
// group of the previous row (in that row's run order) it overlaps by at least `overlap` of the
// shorter of the two, else it opens a group; groups not continued end and are emitted in order.
// Group = (r0, r1, x0, x1).
DEV void wall_group_warp(const uint32_t* runs, const int32_t* cnt, int nrows, int rp, bool transpose, int h, double res, double ox,
                         double oy, int4* act, int4* nxt, uint8_t* used, WallOut& o) {
  const int lane = threadIdx.x & 31;
  int nact = 0;
  int cl = 0;            // lane l holds the run count of row (r & ~31) + l
  unsigned nzm = 0u;     // the rows of that block with runs
  uint32_t myrun = 0u;   // lane q holds run q of the current row
  for (int r = 0; r < nrows; ++r) {
    if ((r & 31) == 0) {   // 32 rows' counts, one load each
      cl = r + lane < nrows ? cnt[r + lane] : 0;
      nzm = __ballot_sync(0xffffffffu, cl != 0);
    }
    if (nact == 0) {   // no group open: on to the next row with runs
      const unsigned rest = nzm & (0xffffffffu << (r & 31));
      if (!rest) {
        r |= 31;
        continue;
      }
      r = (r & ~31) + __ffs(rest) - 1;
    }
    const int nr = __shfl_sync(0xffffffffu, cl, r & 31);
    if (nr == 0 && nact == 0) continue;
    myrun = lane < nr ? runs[(size_t)r * rp + lane] : 0u;   // the row's runs in one load per lane
    for (int i = lane; i < nact; i += 32) used[i] = 0;
    __syncwarp();
    int nn = 0;
    for (int q = 0; q < nr && nn < WALL_ACT_MAX; ++q) {
      const uint32_t rv = q < 32 ? __shfl_sync(0xffffffffu, myrun, q) : runs[(size_t)r * rp + q];
      const int a = (int)(rv & 0xffffu), b = (int)(rv >> 16);
      int hit = -1;
      for (int base = 0; base < nact && hit < 0; base += 32) {
        const int gi = base + lane;
        bool ok = false;
        if (gi < nact && !used[gi]) {
          const int4 g = act[gi];
          if (g.y == r - 1) {
            const int ov = min(b, g.w) - max(a, g.z) + 1;
            ok = (double)ov >= WALL_OVERLAP * (double)min(b - a + 1, g.w - g.z + 1);
          }
        }
        const unsigned msk = __ballot_sync(0xffffffffu, ok);
        if (msk) hit = base + __ffs(msk) - 1;
      }
      if (lane == 0) {
        if (hit < 0) {
          nxt[nn] = make_int4(r, r, a, b);
        } else {
          int4 g = act[hit];
          used[hit] = 1;
          g.y = r;
          g.z = min(g.z, a);
          g.w = max(g.w, b);
          nxt[nn] = g;
        }
      }
      ++nn;
      __syncwarp();
    }
    if (nr > WALL_ACT_MAX && lane == 0) o.ovf = 1;
    if (lane == 0)
      for (int i = 0; i < nact; ++i)
        if (!used[i]) wall_emit(act[i], transpose, h, res, ox, oy, o);
    __syncwarp();
    int4* t = act;
    act = nxt;
    nxt = t;
    nact = nn;
  }
  if (lane == 0)
    for (int i = 0; i < nact; ++i) wall_emit(act[i], transpose, h, res, ox, oy, o);
  __syncwarp();
}

// wallSegments on the bits already built (walls.cpp update: rows first, then columns).  The
// caller's scratch: runs (h * rp_h + w * rp_v), counts (h + w), group lists in shared memory.
DEV void wall_cbits(const uint64_t* bits, int w, int h, int nw, uint64_t* cbits);
DEV void wall_extract(const uint64_t* bits, uint64_t* cbits, int w, int h, int nw, double res, double ox, double oy, uint32_t* runs,
                      int32_t* cnt, unsigned char* smem, WallOut& o, double* vtmp, int* s_ovf) {
  __shared__ int s_hn, s_vn, s_vovf;
  const int min_run = max(1, (int)llround(WALL_MIN_LEN / res));
  const int rp_h = min(w / 2 + 1, WALL_ACT_MAX + 1), rp_v = min(h / 2 + 1, WALL_ACT_MAX + 1);
  uint32_t* hr = runs;
  uint32_t* vr = runs + (size_t)h * rp_h;
  int32_t* hc = cnt;
  int32_t* vc = cnt + h;
  PHASE_START();
  wall_cbits(bits, w, h, nw, cbits);   // columns as rows of bits: their runs are found word-wise too
  wall_row_runs(bits, h, nw, min_run, hr, rp_h, hc, s_ovf);
  __syncthreads();
  PHASE_MARK(56);   // extraction: column bits, row runs
  wall_row_runs(cbits, w, (h + 63) / 64, min_run, vr, rp_v, vc, s_ovf);
  __syncthreads();
  PHASE_MARK(57);   // extraction: column runs
  // rows (warp 0, into o) and columns (warp 1, into vtmp) are chained at the same time; the
  // column segments then follow the row segments, the reference's order
  const int wq = threadIdx.x >> 5;
  if (wq < 2) {
    int4* act = (int4*)smem + (size_t)wq * 2 * WALL_ACT_MAX;
    int4* nxt = act + WALL_ACT_MAX;
    uint8_t* used = (uint8_t*)((int4*)smem + 4 * WALL_ACT_MAX) + (size_t)wq * WALL_ACT_MAX;
    if (wq == 0) {
      wall_group_warp(hr, hc, h, rp_h, false, h, res, ox, oy, act, nxt, used, o);
      if ((threadIdx.x & 31) == 0) s_hn = o.n;
    } else {
      WallOut ov{vtmp, o.cap, 0, 0};
      wall_group_warp(vr, vc, w, rp_v, true, h, res, ox, oy, act, nxt, used, ov);
      if ((threadIdx.x & 31) == 0) { s_vn = ov.n; s_vovf = ov.ovf; }
    }
  }
  __syncthreads();
  PHASE_MARK(58);   // extraction: chaining
  const int hn = s_hn, vn = s_vn;
  for (int i = threadIdx.x; i < 4 * vn; i += blockDim.x)
    if (4 * (size_t)hn + i < 4 * (size_t)o.cap) o.seg[4 * (size_t)hn + i] = vtmp[i];
  if (threadIdx.x == 0) {
    o.n = min(hn + vn, o.cap);
    if (hn + vn > o.cap || s_vovf) o.ovf = 1;
  }
  __syncthreads();
}

// ---- dominant direction (wallAngle) ---------------------------------------------------------

// Projection-histogram scores of angles th[0..na): for each, the sum over bins of squared counts
// of the occupied cells projected on the rotated x and y axes (bins of one cell, float
// arithmetic as the reference's).  A groups of threads each fill their own histograms.
// The occupancy again, column by column (word (x, b) holds rows 64 b .. 64 b + 63 of column x,
// top row first), for the rotated x-axis histogram: its bin changes slowly down a column.
// A warp transposes 32 rows x 64 columns: each lane loads one row's word, 64 ballots give the 64
// columns' 32-bit halves (half g of column x is 32-bit word x * 2 * nwc + g).
DEV void wall_cbits(const uint64_t* bits, int w, int h, int nw, uint64_t* cbits) {
  const int nwc = (h + 63) / 64, lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  uint32_t* c32 = (uint32_t*)cbits;
  for (int t = wid; t < 2 * nwc * nw; t += nwarps) {
    const int g = t / nw, k = t - g * nw, iy = g * 32 + lane;
    const uint64_t v = iy < h ? bits[(size_t)iy * nw + k] : 0ull;
    uint32_t lo = 0u, hi = 0u;
#pragma unroll
    for (int b = 0; b < 64; ++b) {
      const uint32_t col = __ballot_sync(0xffffffffu, (unsigned)((v >> b) & 1ull));
      if (b == lane) lo = col;
      if (b == lane + 32) hi = col;
    }
    const int x0 = k * 64 + lane, x1 = x0 + 32;
    if (x0 < w) c32[(size_t)x0 * 2 * nwc + g] = lo;
    if (x1 < w) c32[(size_t)x1 * 2 * nwc + g] = hi;
  }
}

DEV void wall_scores(const uint64_t* bits, const uint64_t* cbits, int w, int h, int nw, int D, const double* th, int na,
                     unsigned long long* score, int* hist) {
  const int nb = 2 * D + 1;
  const int fit = WALL_SMEM / (int)(2 * nb * sizeof(int));
  const int A = fit >= 8 ? 8 : fit >= 4 ? 4 : fit >= 2 ? 2 : 1;   // whole warps per group
  const int G = blockDim.x / A, grp = threadIdx.x / G, gt = threadIdx.x - grp * G;
  for (int i = threadIdx.x; i < na; i += blockDim.x) score[i] = 0;
  for (int a0 = 0; a0 < na; a0 += A) {
    const int ai = a0 + grp;
    const bool live = grp < A && ai < na;
    int* hx = hist + (size_t)(grp < A ? grp : 0) * 2 * nb;
    int* hy = hx + nb;
    if (grp < A)
      for (int i = gt; i < 2 * nb; i += G) hx[i] = 0;
    __syncthreads();
    if (live) {
      // each bin is counted along the direction it changes slowly in, runs of equal bins in a
      // register: y-axis bins along rows, x-axis bins down columns
      const float c = (float)cos(th[ai]), s = (float)sin(th[ai]), d = __fadd_rn((float)D, 0.5f);
      for (int wi = gt; wi < h * nw; wi += G) {
        uint64_t v = bits[wi];
        if (!v) continue;
        const int iy = wi / nw, k = wi - iy * nw;
        const float py = (float)(h - 1 - iy);
        int pb = -1, pc = 0;
        while (v) {
          const float px = (float)(k * 64 + __ffsll((long long)v) - 1);
          v &= v - 1;
          const int i2 = (int)__fadd_rn(__fadd_rn(__fmul_rn(-s, px), __fmul_rn(c, py)), d);
          if (i2 == pb) {
            ++pc;
          } else {
            if (pc && (unsigned)pb < (unsigned)nb) atomicAdd(&hy[pb], pc);
            pb = i2;
            pc = 1;
          }
        }
        if (pc && (unsigned)pb < (unsigned)nb) atomicAdd(&hy[pb], pc);
      }
      const int nwc = (h + 63) / 64;
      for (int wi = gt; wi < w * nwc; wi += G) {
        uint64_t v = cbits[wi];
        if (!v) continue;
        const int x = wi / nwc, kb = wi - x * nwc;
        const float px = (float)x;
        int pb = -1, pc = 0;
        while (v) {
          const float py = (float)(h - 1 - (kb * 64 + __ffsll((long long)v) - 1));
          v &= v - 1;
          const int i1 = (int)__fadd_rn(__fadd_rn(__fmul_rn(c, px), __fmul_rn(s, py)), d);
          if (i1 == pb) {
            ++pc;
          } else {
            if (pc && (unsigned)pb < (unsigned)nb) atomicAdd(&hx[pb], pc);
            pb = i1;
            pc = 1;
          }
        }
        if (pc && (unsigned)pb < (unsigned)nb) atomicAdd(&hx[pb], pc);
      }
    }
    __syncthreads();
    unsigned long long acc = 0;
    if (live)
      for (int i = gt; i < nb; i += G) acc += (unsigned long long)hx[i] * hx[i] + (unsigned long long)hy[i] * hy[i];
    for (int o = 16; o; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
    if (live && (threadIdx.x & 31) == 0) atomicAdd(&score[ai], acc);
    __syncthreads();
  }
}

// wallAngle (walls.cpp:224-257) on the bits: 1-degree scan of [-45, 45), then 0.25 and 0.05
// degree refinements around the best, folded to [-45, 45) degrees; 0 when fewer than 20 cells are
// occupied or the best beats 0 degrees by less than kAlignGain.
DEV double wall_angle(const uint64_t* bits, uint64_t* cbits, int w, int h, int nw, unsigned char* smem, BlockScratch& bs) {
  __shared__ double s_th[96];
  __shared__ unsigned long long s_sc[96];
  __shared__ double s_best;
  __shared__ unsigned long long s_bv, s_v0;
  int npt = 0;
  for (int i = threadIdx.x; i < h * nw; i += blockDim.x) npt += __popcll(bits[i]);
  npt = block_sum_i(npt, bs);
  if (npt < 20) return 0.0;
  const int D = (int)ceil(hypot((double)w, (double)h)) + 2;
  const double deg = WALL_PI / 180.0;
  if (threadIdx.x == 0) {
    s_th[0] = 0.0;
    for (int k = -45; k < 45; ++k) s_th[1 + k + 45] = k * deg;
  }
  __syncthreads();
  wall_cbits(bits, w, h, nw, cbits);
  __syncthreads();
  wall_scores(bits, cbits, w, h, nw, D, s_th, 91, s_sc, (int*)smem);
  if (threadIdx.x == 0) {
    s_v0 = s_sc[0];
    double best = 0.0;
    unsigned long long bv = s_v0;
    for (int k = 0; k < 90; ++k)
      if (s_sc[1 + k] > bv) { bv = s_sc[1 + k]; best = s_th[1 + k]; }
    s_best = best;
    s_bv = bv;
  }
  __syncthreads();
  for (int stage = 0; stage < 2; ++stage) {
    const double step = stage == 0 ? 0.25 * deg : 0.05 * deg;
    if (threadIdx.x == 0) {
      const double c0 = s_best;
      for (int k = -4; k <= 4; ++k) s_th[k + 4] = c0 + k * step;
    }
    __syncthreads();
    wall_scores(bits, cbits, w, h, nw, D, s_th, 9, s_sc, (int*)smem);
    if (threadIdx.x == 0)
      for (int k = 0; k < 9; ++k)
        if (s_sc[k] > s_bv) { s_bv = s_sc[k]; s_best = s_th[k]; }
    __syncthreads();
  }
  double best = s_best;
  if (best >= WALL_PI / 4) best -= WALL_PI / 2;
  if (best < -WALL_PI / 4) best += WALL_PI / 2;
  if (fabs(best) > WALL_ALIGN_TOL && (double)s_bv < WALL_ALIGN_GAIN * (double)s_v0) return 0.0;
  return best;
}

// ---- tilted maps (wallSegmentsAtAngle, walls.cpp rotatedSegments) ----------------------------

// floor(a / b - off) with a / b the correctly rounded quotient, as the reference computes it:
// from a * (1 / b), whose error is a few ulps, falling back to the division only where that
// product lies within 1e-6 of an integer (there the two floors could differ)
DEV int wall_floor_div(double a, double b, double inv_b, double off) {
  double t = a * inv_b - off;
  if (fabs(t - rint(t)) < 1e-6) t = a / b - off;
  return (int)floor(t);
}

#define WALL_LINES 512     // refined lines of one extraction
#define WALL_PIECES 64     // pieces of one clip
#define WALL_SAMPLES 4096  // samples along one line (half-cell steps)
#define WALL_RPIECES 16    // refined lines one raw segment may leave
#define WALL_RWARPS 16     // warps refining raw segments at once
#define WALL_WSCR 1280     // their shared scratch each: snap profile, sample bits, clip pieces

struct WallLine { int hz; double q, a0, a1; };
static_assert(sizeof(WallLine) == 32, "refined lines are kept in 32-byte slots");

struct WallRot {
  const uint64_t* obits;   // the original window's occupancy (ignore areas cleared), top row first
  int w, h, nw;
  double res, ox, oy, c, s, inv_res;
};

// the original grid's occupancy at the rotated point (u, v) (the cell whose corner is at
// origin + (x, y) * res holds it)
DEV bool wall_occ_uv(const WallRot& G, double u, double v) {
  const double x = G.c * u - G.s * v, y = G.s * u + G.c * v;
  const int ix = wall_floor_div(x - G.ox, G.res, G.inv_res, 0.0), iy = wall_floor_div(y - G.oy, G.res, G.inv_res, 0.0);
  if (ix < 0 || iy < 0 || ix >= G.w || iy >= G.h) return false;
  return (G.obits[(size_t)(G.h - 1 - iy) * G.nw + (ix >> 6)] >> (ix & 63)) & 1ull;
}
DEV bool wall_occ_line(const WallRot& G, const WallLine& l, double t, double d) {
  return l.hz ? wall_occ_uv(G, t, l.q + d) : wall_occ_uv(G, l.q + d, t);
}
DEV int wall_nsamp(const WallRot& G, const WallLine& l) { return max(1, (int)llround((l.a1 - l.a0) / (G.res / 2))); }

// snap (warp): move the line across +-3 cells in quarter-cell steps to the middle of the band
// where its samples are most often occupied; false when the best band is below 0.25
DEV bool wall_snap(const WallRot& G, WallLine& l, double* f) {
  const int lane = threadIdx.x & 31, K = 12, n = wall_nsamp(G, l);
  for (int k = 0; k <= 2 * K; ++k) {
    const double d = (k - K) * G.res / 4;
    int cnt = 0;
    for (int i = lane; i <= n; i += 32) cnt += wall_occ_line(G, l, l.a0 + (l.a1 - l.a0) * i / n, d);
    for (int o = 16; o; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if (lane == 0) f[k] = (double)cnt / (n + 1);
  }
  __syncwarp();
  int ok = 0;
  if (lane == 0) {
    int b = K;
    for (int k = 0; k <= 2 * K; ++k)
      if (f[k] - 0.01 * abs(k - K) > f[b] - 0.01 * abs(b - K)) b = k;
    if (!(f[b] < 0.25)) {
      int lo = b, hi = b;
      while (lo > 0 && f[lo - 1] >= 0.5 * f[b]) --lo;
      while (hi < 2 * K && f[hi + 1] >= 0.5 * f[b]) ++hi;
      double sw = 0, sd = 0;
      for (int k = lo; k <= hi; ++k) { sw += f[k]; sd += f[k] * (k - K) * G.res / 4; }
      l.q += sd / sw;
      ok = 1;
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  l.q = __shfl_sync(0xffffffffu, l.q, 0);
  return ok;
}

// clip (warp): split the line where occupancy (within half a cell across it) breaks for more
// than 4 cells and trim its ends to occupied samples; keep pieces of min_len (less a cell) at
// least 70 % occupied.  Returns the number of pieces (lane 0's list).
DEV int wall_clip(const WallRot& G, const WallLine& l, uint32_t* onw, WallLine* out, int pcap, int* ovf) {
  const int lane = threadIdx.x & 31, n = wall_nsamp(G, l);
  if (n + 1 > WALL_SAMPLES) { if (lane == 0) *ovf = 1; return 0; }
  const double hr = G.res / 2;
  for (int i0 = 0; i0 <= n; i0 += 32) {   // occupancy of the samples as bits, 32 by a ballot
    const int i = i0 + lane;
    bool v = false;
    if (i <= n) {
      const double t = l.a0 + (l.a1 - l.a0) * i / n;
      v = wall_occ_line(G, l, t, 0) || wall_occ_line(G, l, t, -hr) || wall_occ_line(G, l, t, hr);
    }
    const unsigned bal = __ballot_sync(0xffffffffu, v);
    if (lane == 0) onw[i0 >> 5] = bal;
  }
  __syncwarp();
  int np = 0;
  if (lane == 0) {
    int first = -1, last = -1, cnt = 0, gap = 0;
    auto close = [&]() {
      if (first >= 0) {
        const double t0 = l.a0 + (l.a1 - l.a0) * first / n, t1 = l.a0 + (l.a1 - l.a0) * last / n;
        if (t1 - t0 >= WALL_MIN_LEN - G.res - 1e-9 && (double)cnt >= 0.7 * (last - first + 1)) {
          if (np < pcap) out[np++] = WallLine{l.hz, l.q, t0, t1};
          else *ovf = 1;
        }
      }
      first = last = -1;
      cnt = 0;
      gap = 0;
    };
    for (int i = 0; i <= n; ++i) {
      if ((onw[i >> 5] >> (i & 31)) & 1u) {
        if (first < 0) first = i;
        last = i;
        ++cnt;
        gap = 0;
      } else if (first >= 0 && ++gap > 8) {
        close();
      }
    }
    close();
  }
  np = __shfl_sync(0xffffffffu, np, 0);
  __syncwarp();
  return np;
}

// refine (warp): snap, clip, snap every piece; appends to out (lane 0), returns the count added
DEV int wall_refine(const WallRot& G, WallLine l, double* f, uint32_t* onw, WallLine* pcs, int pcap, WallLine* out, int cap, int* ovf) {
  if (!wall_snap(G, l, f)) return 0;
  const int np = wall_clip(G, l, onw, pcs, pcap, ovf);
  int added = 0;
  for (int p = 0; p < np; ++p) {
    WallLine q = pcs[p];
    __syncwarp();
    if (wall_snap(G, q, f)) {
      if ((threadIdx.x & 31) == 0) {
        if (added < cap) out[added] = q;
        else *ovf = 1;
      }
      ++added;
    }
  }
  __syncwarp();
  return min(added, cap);
}

DEV void wall_refit_warp(const Batch& B, int m, const WallRot& G, const double* raw, int nraw, unsigned char* smem, int* s_ovf);

// wallSegmentsAtAngle for |th| > kAlignTol: the window rotated by -th (a rotated cell is occupied
// when any of the four original cells around its centre is), axis-aligned extraction there, each
// segment refitted to the original occupancy (snap, clip, snap), nearby collinear lines merged and
// refitted, short lines shadowed by a longer parallel one dropped, and the rest rotated back.
DEV void wall_tilted(const Batch& B, int m, const int8_t* cells, uint64_t* obits, const int4* rc0, const int4* rc1, int nrc, double th,
                     unsigned char* smem, BlockScratch& bs, int* s_ovf) {
  (void)cells; (void)bs;
  PHASE_START();
  const int w = B.gw_grid, h = B.gh_grid, nw = (w + 63) / 64;
  const double res = (double)B.p.grid_res, ox = B.gx0 * res, oy = B.gy0 * res;
  wall_bits(cells, w, h, nw, obits, rc0, rc1, nrc);   // the masked source (maskIgnore)
  const double c = cos(th), s = sin(th);
  double u0 = 1e300, v0 = 1e300, u1 = -1e300, v1 = -1e300;
  for (int k = 0; k < 4; ++k) {
    const double x = ox + ((k & 1) ? w : 0) * res, y = oy + ((k & 2) ? h : 0) * res;
    const double u = c * x + s * y, v = -s * x + c * y;
    u0 = smin(u0, u); u1 = smax(u1, u); v0 = smin(v0, v); v1 = smax(v1, v);
  }
  const int RW = (int)ceil((u1 - u0) / res) + 1, RH = (int)ceil((v1 - v0) / res) + 1, rnw = (RW + 63) / 64;
  if (RW > B.wscr_side || RH > B.wscr_side) {
    if (threadIdx.x == 0) *s_ovf = 1;
    return;
  }
  __syncthreads();
  PHASE_MARK(50);   // tilted: masked source bits
  const double inv_res = 1.0 / res;
  // rotated occupancy bits, top row first.  A rotated cell is occupied when any of the four
  // original cells (x0 .. x0 + 1, y0 .. y0 + 1) around its centre is: the 2 x 2 dilation D of the
  // occupancy answers that with one lookup, D(x0, y0) at bit x0 + 1 of row y0 + 1 (x0, y0 from -1,
  // cells outside the window unoccupied), kept in shared memory when it fits (37 KB for 512 x 512)
  uint64_t* rbits = obits + (size_t)B.wbits_half;
  const int dnw = (w + 1 + 63) / 64, drows = h + 1;
  // (else in the column-bit area, free until the extraction on the rotated grid)
  uint64_t* D = (size_t)drows * dnw * 8 <= (size_t)WALL_SMEM ? (uint64_t*)smem : obits + B.wbits_cb;
  for (int t = threadIdx.x; t < drows * dnw; t += blockDim.x) {
    const int r = t / dnw, k = t - r * dnw, y0 = r - 1;
    // E_y(b) = A_y(b - 1) | A_y(b): A_y = the occupancy of grid row y (bit x), shifted by one
    auto row_e = [&](int y) -> uint64_t {
      if (y < 0 || y >= h) return 0ull;
      const uint64_t* A = obits + (size_t)(h - 1 - y) * nw;
      const uint64_t a = k < nw ? A[k] : 0ull, ap = k > 0 && k - 1 < nw ? A[k - 1] : 0ull;
      const uint64_t sh = (a << 1) | (ap >> 63);   // bit b = A(b - 1)
      return sh | a;
    };
    D[t] = row_e(y0) | row_e(y0 + 1);
  }
  __syncthreads();
  // The cell centre in original cells is affine in the rotated cell (i, j): fx = c (i + 1/2) -
  // s (j + 1/2) + Kx, fy = s (i + 1/2) + c (j + 1/2) + Ky.  Its floor comes from that form in
  // float (error below 1e-6 of the terms' magnitude); the reference's double expression is
  // evaluated only where the float value lies closer than that to an integer.
  const float cf = (float)c, sf = (float)s;
  const float Kx = (float)((c * u0 - s * v0 - ox) * inv_res - 0.5), Ky = (float)((s * u0 + c * v0 - oy) * inv_res - 0.5);
  for (int i = threadIdx.x; i < RH * rnw; i += blockDim.x) {
    const int iy = i / rnw, k = i - iy * rnw, j = RH - 1 - iy;
    const double v = v0 + (j + 0.5) * res;
    const float jf = (float)j + 0.5f;
    uint64_t word = 0;
    for (int b = 0; b < 64 && k * 64 + b < RW; ++b) {
      const float if_ = (float)(k * 64 + b) + 0.5f;
      const float ax = cf * if_, bx = sf * jf, ay = sf * if_, by = cf * jf;
      const float fxf = ax - bx + Kx, fyf = ay + by + Ky;
      const float ex = 1e-6f * (fabsf(ax) + fabsf(bx) + fabsf(Kx) + 1.f), ey = 1e-6f * (fabsf(ay) + fabsf(by) + fabsf(Ky) + 1.f);
      int x0, y0;
      if (fabsf(fxf - rintf(fxf)) > ex && fabsf(fyf - rintf(fyf)) > ey) {
        x0 = (int)floorf(fxf);
        y0 = (int)floorf(fyf);
      } else {
        const double u = u0 + (k * 64 + b + 0.5) * res;
        x0 = wall_floor_div(c * u - s * v - ox, res, inv_res, 0.5);
        y0 = wall_floor_div(s * u + c * v - oy, res, inv_res, 0.5);
      }
      bool occ = false;
      if (x0 >= -1 && x0 < w && y0 >= -1 && y0 < h) {
        const int bx1 = x0 + 1;
        occ = (D[(size_t)(y0 + 1) * dnw + (bx1 >> 6)] >> (bx1 & 63)) & 1ull;
      }
      word |= (uint64_t)occ << b;
    }
    rbits[i] = word;
  }
  __syncthreads();
  PHASE_MARK(51);   // tilted: rotated bits
  // raw segments on the rotated grid (coordinates u, v)
  double* raw = B.wall_raw + (size_t)m * SMG_WALL_SEGS_MAX * 4;
  WallOut o{raw, SMG_WALL_SEGS_MAX, 0, 0};
  uint32_t* runs = B.wruns + (size_t)m * B.wruns_stride;
  int32_t* cnt = (int32_t*)(rc1 + B.O);
  wall_extract(rbits, obits + B.wbits_cb, RW, RH, rnw, res, u0, v0, runs, cnt, smem, o, B.wall_tmp + (size_t)m * SMG_WALL_SEGS_MAX * 4,
               s_ovf);
  PHASE_MARK(52);   // tilted: extraction on the rotated grid
  __shared__ int s_nraw;
  if (threadIdx.x == 0) {
    s_nraw = o.n;
    if (o.ovf) *s_ovf = 1;
  }
  // the original occupancy in shared memory when it fits beside the lists (a 512 x 512 window
  // takes 32 KB): the samples' reads then wait for no global load
  const uint64_t* ob = obits;
  if ((size_t)32768 + (size_t)h * nw * 8 <= (size_t)65536) {
    uint64_t* sob = (uint64_t*)(smem + 32768);
    for (int i = threadIdx.x; i < h * nw; i += blockDim.x) sob[i] = obits[i];
    ob = sob;
  }
  __syncthreads();
  const WallRot G{ob, w, h, nw, res, ox, oy, c, s, inv_res};
  // refine the raw segments (independent of one another), WALL_RWARPS warps at once; each
  // leaves its lines in the segment's slot
  const int nraw = s_nraw, wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (wid < WALL_RWARPS) {
    unsigned char* ws = smem + 65536 + (size_t)wid * WALL_WSCR;
    double* f = (double*)ws;
    uint32_t* onw = (uint32_t*)(ws + 256);
    WallLine* pcs = (WallLine*)(ws + 768);
    for (int r = wid; r < nraw; r += WALL_RWARPS) {
      const double* q = raw + 4 * r;
      const bool hz = q[1] == q[3];
      const WallLine l = hz ? WallLine{1, q[1], smin(q[0], q[2]), smax(q[0], q[2])} : WallLine{0, q[0], smin(q[1], q[3]), smax(q[1], q[3])};
      WallLine* outl = (WallLine*)B.wall_lines + ((size_t)m * SMG_WALL_SEGS_MAX + r) * WALL_RPIECES;
      const int k = wall_refine(G, l, f, onw, pcs, (WALL_WSCR - 768) / (int)sizeof(WallLine), outl, WALL_RPIECES, s_ovf);
      if (lane == 0) B.wall_lcnt[(size_t)m * SMG_WALL_SEGS_MAX + r] = k;
    }
  }
  __syncthreads();
  PHASE_MARK(53);   // refit: the raw segments refined
  if (threadIdx.x < 32) wall_refit_warp(B, m, G, raw, nraw, smem, s_ovf);
  __syncthreads();
}

// The rest of rotatedSegments by one warp: the refined lines in raw order, merges, shadows and
// the rotation back.  Shared memory (below the staged occupancy) holds the lines, clip pieces,
// the sample bits and the snap profile.
DEV void wall_refit_warp(const Batch& B, int m, const WallRot& G, const double* raw, int nraw, unsigned char* smem, int* s_ovf) {
  MapRec* R = &B.maps[m];
  const int lane = threadIdx.x;
  const double res = G.res, c = G.c, s = G.s;
  PHASE_START();
  (void)raw;
  WallLine* lines = (WallLine*)smem;
  WallLine* pcs = lines + WALL_LINES;
  WallLine* tmp = pcs + WALL_PIECES;
  double* f = (double*)(tmp + WALL_PIECES);
  uint32_t* on = (uint32_t*)(f + 32);
  int nl = 0;
  for (int r = 0; r < nraw; ++r) {   // the segments' lines, in the raw segments' order
    const int k = B.wall_lcnt[(size_t)m * SMG_WALL_SEGS_MAX + r];
    const WallLine* src = (const WallLine*)B.wall_lines + ((size_t)m * SMG_WALL_SEGS_MAX + r) * WALL_RPIECES;
    for (int i = lane; i < k; i += 32)
      if (nl + i < WALL_LINES) lines[nl + i] = src[i];
    if (nl + k > WALL_LINES && lane == 0) *s_ovf = 1;
    nl = min(nl + k, WALL_LINES);
  }
  __syncwarp();
  // merge collinear neighbours until none is left (the first pair in (i, j) order each time);
  // every merge leaves fewer lines or pieces more than 4 cells apart, the guard only bounds a
  // damaged list
  for (int guard = 0;; ++guard) {
    if (guard >= 4 * WALL_LINES) {
      if (lane == 0) *s_ovf = 1;
      break;
    }
    // the first mergeable pair in (i, j) order: for each i, the lanes test 32 j at a time
    int pi = -1, pj = -1;
    for (int i = 0; i < nl && pi < 0; ++i) {
      const WallLine a = lines[i];
      for (int j0 = i + 1; j0 < nl; j0 += 32) {
        const int j = j0 + lane;
        bool ok = false;
        if (j < nl) {
          const WallLine& b = lines[j];
          ok = !(a.hz != b.hz || fabs(a.q - b.q) > 2 * res + 1e-9 || smin(a.a1, b.a1) - smax(a.a0, b.a0) < -res - 1e-9);
        }
        const unsigned msk = __ballot_sync(0xffffffffu, ok);
        if (msk) {
          pi = i;
          pj = j0 + __ffs(msk) - 1;
          break;
        }
      }
    }
    if (pi < 0) break;
    const WallLine a = lines[pi], b = lines[pj];
    const double la = a.a1 - a.a0 + res, lb = b.a1 - b.a0 + res;
    const WallLine mg{a.hz, (a.q * la + b.q * lb) / (la + lb), smin(a.a0, b.a0), smax(a.a1, b.a1)};
    const int np = wall_refine(G, mg, f, on, pcs, WALL_PIECES, tmp, WALL_PIECES, s_ovf);
    if (lane == 0) {
      // erase j, erase i, insert the pieces at i
      for (int k = pj; k + 1 < nl; ++k) lines[k] = lines[k + 1];
      --nl;
      for (int k = pi; k + 1 < nl; ++k) lines[k] = lines[k + 1];
      --nl;
      const int room = min(np, WALL_LINES - nl);
      if (room < np) *s_ovf = 1;
      for (int k = nl - 1; k >= pi; --k) lines[k + room] = lines[k];
      for (int k = 0; k < room; ++k) lines[pi + k] = tmp[k];
      nl += room;
    }
    nl = __shfl_sync(0xffffffffu, nl, 0);
    __syncwarp();
  }
  PHASE_MARK(54);   // refit: merges
  // to segments, drop shadowed short parallels, rotate back into the map frame
  double* Wl = B.wall_w + (size_t)m * SMG_WALL_SEGS_MAX * 4;
  if (lane == 0) {
    const double tol = WALL_MAX_THICK / 2, slack = res;
    auto seg = [&](int i, double* q) {
      const WallLine& l = lines[i];
      if (l.hz) { q[0] = l.a0; q[1] = l.q; q[2] = l.a1; q[3] = l.q; }
      else { q[0] = l.q; q[1] = l.a0; q[2] = l.q; q[3] = l.a1; }
    };
    int n = 0;
    for (int i = 0; i < nl; ++i) {
      double a[4];
      seg(i, a);
      const bool ha = a[1] == a[3];
      const double alen = ha ? fabs(a[2] - a[0]) : fabs(a[3] - a[1]);
      const double a0 = ha ? smin(a[0], a[2]) : smin(a[1], a[3]), a1 = ha ? smax(a[0], a[2]) : smax(a[1], a[3]);
      bool shadow = false;
      for (int j = 0; j < nl && !shadow; ++j) {
        double b[4];
        seg(j, b);
        if (j == i || (b[1] == b[3]) != ha) continue;
        const double blen = ha ? fabs(b[2] - b[0]) : fabs(b[3] - b[1]);
        if (blen < alen || (blen == alen && j > i)) continue;
        const double off = ha ? fabs(a[1] - b[1]) : fabs(a[0] - b[0]);
        const double b0 = ha ? smin(b[0], b[2]) : smin(b[1], b[3]), b1 = ha ? smax(b[0], b[2]) : smax(b[1], b[3]);
        shadow = off <= tol && a0 >= b0 - slack && a1 <= b1 + slack;
      }
      if (shadow) continue;
      if (n >= SMG_WALL_SEGS_MAX) { *s_ovf = 1; break; }
      double* q = Wl + 4 * (size_t)n++;
      q[0] = c * a[0] - s * a[1];
      q[1] = s * a[0] + c * a[1];
      q[2] = c * a[2] - s * a[3];
      q[3] = s * a[2] + c * a[3];
    }
    R->n_w = n;
  }
  __syncwarp();
  PHASE_MARK(55);   // refit: shadows, rotation back
}

// ---- the keyframe's wall list ---------------------------------------------------------------

// The window bridges (capi.cpp:873-887): for segment pairs i < j (in order) on one line (parallel
// within 0.03, 0.1 m apart), the gap between them when shorter than bridge_max.  Thread per i
// counts, a scan orders, the same thread writes.
DEV int wall_bridge(const double* W, int i, int j, double bmax, double* out) {
  const double* A = W + 4 * i;
  const double* Bj = W + 4 * j;
  const double ux = A[2] - A[0], uy = A[3] - A[1], li = hypot(ux, uy);
  const double vx = Bj[2] - Bj[0], vy = Bj[3] - Bj[1], lj = hypot(vx, vy);
  if (li < 1e-6 || lj < 1e-6 || fabs(ux * vy - uy * vx) / (li * lj) > 0.03) return 0;
  const double nx = -uy / li, ny = ux / li;
  if (fabs((Bj[0] - A[0]) * nx + (Bj[1] - A[1]) * ny) > 0.1) return 0;
  const double a0 = 0, a1 = li;
  double b0 = ((Bj[0] - A[0]) * ux + (Bj[1] - A[1]) * uy) / li, b1 = ((Bj[2] - A[0]) * ux + (Bj[3] - A[1]) * uy) / li;
  if (b0 > b1) { const double t = b0; b0 = b1; b1 = t; }
  const double lo = a1 <= b0 ? a1 : b1, hi = a1 <= b0 ? b0 : a0;
  if (hi - lo <= 0 || hi - lo > bmax) return 0;
  if (out) {
    out[0] = A[0] + ux / li * lo;
    out[1] = A[1] + uy / li * lo;
    out[2] = A[0] + ux / li * hi;
    out[3] = A[1] + uy / li * hi;
  }
  return 1;
}

__global__ void __launch_bounds__(WALL_THREADS) k_walls(Batch B) {
  extern __shared__ __align__(16) unsigned char wl_smem[];
  __shared__ BlockScratch bs;
  __shared__ int s_angle, s_mode, s_ovf, s_scan[2][33];
  __shared__ double s_thn;
  const int m = B.map0 + blockIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active || !B.walls_on) return;
  MapRec* R = &B.maps[m];
  const int w = B.gw_grid, h = B.gh_grid, nw = (w + 63) / 64;
  const double res = (double)B.p.grid_res, ox = B.gx0 * res, oy = B.gy0 * res;
  const double now = F.stamp;
  const size_t O = (size_t)B.O;
  if (threadIdx.x == 0) {
    const bool grid_changed = R->w_dirty, rchg = R->w_rchg;
    s_angle = (grid_changed || rchg) && now - R->w_th_t >= WALL_ANGLE_EVERY;
    s_ovf = 0;
  }
  __syncthreads();
  // the ignore rectangles as cell ranges (walls.cpp maskIgnore / update)
  const int nrc = R->n_rect;
  int4* rc0 = (int4*)(B.wscr_i + (size_t)m * B.wscr_i_stride);
  int4* rc1 = rc0 + O;
  const double* rect = B.wrect + (size_t)m * O * 4;
  for (int r = threadIdx.x; r < nrc; r += blockDim.x) {
    const double* q = rect + 4 * r;
    rc0[r] = make_int4(max(0, (int)floor((q[0] - ox) / res)), max(0, (int)floor((q[1] - oy) / res)), 0, 0);
    rc1[r] = make_int4(min(w - 1, (int)floor((q[2] - ox) / res)), min(h - 1, (int)floor((q[3] - oy) / res)), 0, 0);
  }
  __syncthreads();
  uint64_t* bits = B.wbits + (size_t)m * B.wbits_stride;
  const int8_t* cells = B.gc8 + (size_t)m * w * h;
  bool built = false;
  if (s_angle) {
    wall_bits(cells, w, h, nw, bits, rc0, rc1, nrc);
    __syncthreads();
    built = true;
    const double th = wall_angle(bits, bits + B.wbits_cb, w, h, nw, wl_smem, bs);
    if (threadIdx.x == 0) s_thn = th;
  }
  if (threadIdx.x == 0) {
    const bool grid_changed = R->w_dirty, rchg = R->w_rchg;
    bool th_changed = false;
    if (s_angle) {
      const double th = s_thn;
      R->w_th_t = now;
      if (fabs(th - R->w_th) > WALL_ANGLE_HYST) {
        const bool was_axis = fabs(R->w_th) <= WALL_ALIGN_TOL, is_axis = fabs(th) <= WALL_ALIGN_TOL;
        if (was_axis != is_axis) R->w_has = 0;
        R->w_th = th;
        th_changed = true;
      }
    }
    if (fabs(R->w_th) > WALL_ALIGN_TOL)
      s_mode = (R->w_has && !th_changed && !rchg && (!grid_changed || now - R->w_full_t < WALL_ALIGNED_EVERY)) ? 0 : 2;
    else
      s_mode = (R->w_has && !grid_changed && !rchg) ? 0 : 1;
  }
  __syncthreads();
  double* Wl = B.wall_w + (size_t)m * SMG_WALL_SEGS_MAX * 4;
  if (s_mode == 1) {
    if (!built) {
      wall_bits(cells, w, h, nw, bits, rc0, rc1, nrc);
      __syncthreads();
    }
    WallOut o{Wl, SMG_WALL_SEGS_MAX, 0, 0};
    uint32_t* runs = B.wruns + (size_t)m * B.wruns_stride;
    int32_t* cnt = (int32_t*)(rc1 + O);
    wall_extract(bits, bits + B.wbits_cb, w, h, nw, res, ox, oy, runs, cnt, wl_smem, o, B.wall_tmp + (size_t)m * SMG_WALL_SEGS_MAX * 4,
                 &s_ovf);
    if (threadIdx.x == 0) {
      R->n_w = o.n;
      if (o.ovf) s_ovf = 1;
    }
  } else if (s_mode == 2) {
    // tilted maps: wallSegmentsAtAngle
    wall_tilted(B, m, cells, bits, rc0, rc1, nrc, R->w_th, wl_smem, bs, &s_ovf);
  }
  if (s_mode != 0) {
    double* prev = B.wrect_prev + (size_t)m * O * 4;
    for (int i = threadIdx.x; i < 4 * nrc; i += blockDim.x) prev[i] = rect[i];
    if (threadIdx.x == 0) {
      R->n_rect_prev = nrc;
      R->w_has = 1;
      R->w_dirty = 0;
      if (s_mode == 2) R->w_full_t = now;
    }
  }
  __syncthreads();
  // the keyframe's list: the segments, then the bridges (an empty list leaves the stored set)
  const int nW = R->w_has ? R->n_w : 0;
  const double bmax = B.p.bridge_max;
  double* out = B.wsegs + (size_t)m * SMG_WALL_SEGS_MAX * 4;
  for (int i = threadIdx.x; i < 4 * nW; i += blockDim.x) out[i] = Wl[i];
  int before = nW, it = 0;
  for (int i0 = 0; i0 < nW; i0 += blockDim.x) {
    const int i = i0 + threadIdx.x;
    int nb = 0;
    if (i < nW && bmax > 0)
      for (int j = i + 1; j < nW; ++j) nb += wall_bridge(Wl, i, j, bmax, nullptr);
    int tot;
    int at = before + block_scan_db(nb, &tot, s_scan, it++);
    if (nb)
      for (int j = i + 1; j < nW; ++j) {
        double q[4];
        if (!wall_bridge(Wl, i, j, bmax, q)) continue;
        if (at < SMG_WALL_SEGS_MAX)
          for (int c = 0; c < 4; ++c) out[4 * (size_t)at + c] = q[c];
        ++at;
      }
    before += tot;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int total = min(before, SMG_WALL_SEGS_MAX);
    if (before > SMG_WALL_SEGS_MAX || s_ovf) set_err(R, SMG_E_CAP_WALLS);
    R->wfr = total;
    if (total > 0) R->n_wseg = total;
  }
}

// ---- the wall state of a pose (sm_snap_wall_state) --------------------------------------------

// rayDistances (walls.cpp:427-453): 16 rays from the pose, first occupied window cell by grid
// traversal (Amanatides and Woo), distance or max_range; segmentsRobotFrame (:455-478): the 8
// nearest segments in the robot frame; wallStateVector (:480-490).  One CTA.
__global__ void __launch_bounds__(256) k_wall_state(Batch B, int m, double px, double py, double yaw, float* out) {
  __shared__ double s_d[SMG_WALL_SEGS_MAX];
  __shared__ float s_rays[WALL_SECTORS];
  const MapRec& R = B.maps[m];
  const int w = B.gw_grid, h = B.gh_grid;
  const double res = (double)B.p.grid_res, ox = B.gx0 * res, oy = B.gy0 * res;
  const int8_t* cells = B.gc8 + (size_t)m * w * h;
  if (threadIdx.x < WALL_SECTORS) {
    const int i = threadIdx.x;
    const double th = yaw + 2.0 * WALL_PI * i / WALL_SECTORS;
    const double dx = cos(th), dy = sin(th);
    const double fx = (px - ox) / res, fy = (py - oy) / res;
    int cx = (int)floor(fx), cy = (int)floor(fy);
    const int sx = dx > 0 ? 1 : -1, sy = dy > 0 ? 1 : -1;
    const double inf = __longlong_as_double(0x7ff0000000000000ll);
    const double tdx = dx != 0 ? fabs(res / dx) : inf, tdy = dy != 0 ? fabs(res / dy) : inf;
    double tx = dx != 0 ? ((sx > 0 ? cx + 1 - fx : fx - cx) * res) / fabs(dx) : inf;
    double ty = dy != 0 ? ((sy > 0 ? cy + 1 - fy : fy - cy) * res) / fabs(dy) : inf;
    float best = (float)WALL_MAX_RANGE;
    double t = 0;
    for (int guard = 0; t <= WALL_MAX_RANGE && guard < 4 * (w + h) + 8; ++guard) {
      if (cx >= 0 && cx < w && cy >= 0 && cy < h && cells[(size_t)cy * w + cx] >= WALL_OCC) {
        best = (float)smax(t, 0.0);
        break;
      }
      if (tx < ty) { t = tx; tx += tdx; cx += sx; }
      else { t = ty; ty += tdy; cy += sy; }
    }
    s_rays[i] = best;
  }
  const int n = R.w_has ? R.n_w : 0;
  const double* W = B.wall_w + (size_t)m * SMG_WALL_SEGS_MAX * 4;
  const double c = cos(-yaw), s = sin(-yaw);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const double* q = W + 4 * i;
    const double ax = q[0] - px, ay = q[1] - py, bx = q[2] - px, by = q[3] - py;
    const double rax = c * ax - s * ay, ray = s * ax + c * ay, rbx = c * bx - s * by, rby = s * bx + c * by;
    const double abx = rbx - rax, aby = rby - ray;
    double t = -(rax * abx + ray * aby) / smax(abx * abx + aby * aby, 1e-12);
    t = t < 0.0 ? 0.0 : (1.0 < t ? 1.0 : t);
    s_d[i] = hypot(rax + abx * t, ray + aby * t);
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  for (int i = 0; i < WALL_SECTORS; ++i) out[i] = (float)(s_rays[i] / WALL_MAX_RANGE);
  // the k nearest, nearest first (ties: the earlier segment)
  const int k = min(WALL_SEGMENTS, n);
  int taken[WALL_SEGMENTS];
  for (int j = 0; j < WALL_SEGMENTS; ++j) {
    float* o = out + WALL_SECTORS + 5 * j;
    int bi = -1;
    if (j < k)
      for (int i = 0; i < n; ++i) {
        bool used = false;
        for (int q = 0; q < j; ++q) used = used || taken[q] == i;
        if (!used && (bi < 0 || s_d[i] < s_d[bi])) bi = i;
      }
    if (j < WALL_SEGMENTS) taken[j] = bi;
    const float dist = bi >= 0 ? (float)s_d[bi] : __int_as_float(0x7f800000);
    const bool valid = isfinite(dist) && dist <= WALL_MAX_RANGE * 1.5;
    if (!valid || bi < 0) {
      for (int q = 0; q < 5; ++q) o[q] = 0.f;
      continue;
    }
    const double* q = W + 4 * bi;
    const double ax = q[0] - px, ay = q[1] - py, bx = q[2] - px, by = q[3] - py;
    const float seg[4] = {(float)(c * ax - s * ay), (float)(s * ax + c * ay), (float)(c * bx - s * by), (float)(s * bx + c * by)};
    for (int e = 0; e < 4; ++e) {
      const float v = (float)(seg[e] / WALL_MAX_RANGE);
      o[e] = v < -1.f ? -1.f : (1.f < v ? 1.f : v);
    }
    o[4] = 1.f;
  }
}
