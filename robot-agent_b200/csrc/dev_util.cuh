// Device helpers: block-wide reductions / scans / exact k-th selection, hashing, and the
// scalar formulas of the reference's objprob math (scenemap include/scenemap/objprob_math.h)
// restated for the device.  Compiled with --fmad=false so that every float/double expression
// rounds exactly like the reference's host build (baseline x86-64, no FMA contraction).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "smg_internal.h"

#define DEV __device__ __forceinline__

// Phase timing (instrumentation builds only, -DSMG_PHASE_TIMING): thread 0 of a block adds the
// clock cycles since its previous mark to phase slot i (smg_phase_read).  No-ops otherwise.
#ifdef SMG_PHASE_TIMING
__device__ unsigned long long g_phase_cycles[64];
__device__ unsigned long long g_phase_hits[64];
#define PHASE_START() long long phase_t_ = clock64()
#define PHASE_MARK(i)                                                              \
  do {                                                                             \
    if (threadIdx.x == 0) {                                                        \
      const long long n_ = clock64();                                              \
      atomicAdd(&g_phase_cycles[(i)], (unsigned long long)(n_ - phase_t_));        \
      atomicAdd(&g_phase_hits[(i)], 1ull);                                         \
      phase_t_ = n_;                                                               \
    }                                                                              \
  } while (0)
#define PHASE_COUNT(i)                                                             \
  do {                                                                             \
    if (threadIdx.x == 0) atomicAdd(&g_phase_hits[(i)], 1ull);                     \
  } while (0)
#else
#define PHASE_START() do { } while (0)
#define PHASE_MARK(i) do { } while (0)
#define PHASE_COUNT(i) do { } while (0)
#endif

// Self-checks (built with -DSMG_CHECKS): an index outside [0, n) records (site, index, bound) of
// the first failure in smg_chk and the access is skipped.  Without SMG_CHECKS they compile away.
__device__ unsigned long long smg_chk[3];
#ifdef SMG_CHECKS
__device__ __noinline__ bool smg_chk_fail(int site, long long i, long long n) {
  if (atomicCAS(&smg_chk[0], 0ull, (unsigned long long)site) == 0ull) {
    smg_chk[1] = (unsigned long long)i;
    smg_chk[2] = (unsigned long long)n;
  }
  return false;
}
#define INB(i, n, site) (((long long)(i) >= 0 && (long long)(i) < (long long)(n)) ? true : smg_chk_fail(site, (long long)(i), (long long)(n)))
#else
#define INB(i, n, site) true
#endif

// ---------------------------------------------------------------- block primitives
// All helpers assume blockDim.x is a multiple of 32 and <= 1024, and that every thread of the
// block calls them (they contain __syncthreads).

struct BlockScratch {
  double d[32];
  long long ll[32];
  int i[33];
};

DEV double warp_sum_d(double v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
DEV long long warp_sum_ll(long long v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
DEV int warp_sum_i(int v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
DEV double warp_max_d(double v) {
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
DEV double warp_min_d(double v) {
  for (int o = 16; o > 0; o >>= 1) v = fmin(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// deterministic block sum (fixed tree for a given blockDim)
DEV double block_sum_d(double v, BlockScratch& s) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum_d(v);
  __syncthreads();
  if (lane == 0) s.d[wid] = v;
  __syncthreads();
  double r = 0;
  if (wid == 0) {
    r = lane < nw ? s.d[lane] : 0.0;
    r = warp_sum_d(r);
    if (lane == 0) s.d[0] = r;
  }
  __syncthreads();
  r = s.d[0];
  __syncthreads();
  return r;
}
DEV long long block_sum_ll(long long v, BlockScratch& s) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum_ll(v);
  __syncthreads();
  if (lane == 0) s.ll[wid] = v;
  __syncthreads();
  long long r = 0;
  if (wid == 0) {
    r = lane < nw ? s.ll[lane] : 0;
    r = warp_sum_ll(r);
    if (lane == 0) s.ll[0] = r;
  }
  __syncthreads();
  r = s.ll[0];
  __syncthreads();
  return r;
}
DEV int block_sum_i(int v, BlockScratch& s) { return (int)block_sum_ll(v, s); }
DEV double block_max_d(double v, BlockScratch& s) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max_d(v);
  __syncthreads();
  if (lane == 0) s.d[wid] = v;
  __syncthreads();
  double r = -1e308;
  if (wid == 0) {
    r = lane < nw ? s.d[lane] : -1e308;
    r = warp_max_d(r);
    if (lane == 0) s.d[0] = r;
  }
  __syncthreads();
  r = s.d[0];
  __syncthreads();
  return r;
}
DEV double block_min_d(double v, BlockScratch& s) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_min_d(v);
  __syncthreads();
  if (lane == 0) s.d[wid] = v;
  __syncthreads();
  double r = 1e308;
  if (wid == 0) {
    r = lane < nw ? s.d[lane] : 1e308;
    r = warp_min_d(r);
    if (lane == 0) s.d[0] = r;
  }
  __syncthreads();
  r = s.d[0];
  __syncthreads();
  return r;
}

// N sums in one reduction (deterministic tree); buf: N*32 shared doubles.
template <int N>
DEV void block_sum_multi(double (&v)[N], double* buf) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int k = 0; k < N; ++k) v[k] = warp_sum_d(v[k]);
  if (lane == 0)
    for (int k = 0; k < N; ++k) buf[k * 32 + wid] = v[k];
  __syncthreads();
  for (int k = 0; k < N; ++k) {   // every thread adds the warp sums in warp order
    double r = 0.0;
    for (int w = 0; w < nw; ++w) r += buf[k * 32 + w];
    v[k] = r;
  }
  __syncthreads();
}

// Exclusive scan of a 0/1 (or small int) flag across the block; returns the prefix for this
// thread and writes the block total to *total.  Order = thread order (used for ordered
// stream compaction: chunk c covers elements c*blockDim .. c*blockDim+blockDim-1).
DEV int block_excl_scan(int flag, int* total, BlockScratch& s) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = flag;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31 && INB(wid, 33, 131)) s.i[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int w = lane < nw ? s.i[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) s.i[lane] = w;   // inclusive per-warp totals
  }
  __syncthreads();
  const int before = wid > 0 ? s.i[wid - 1] : 0;
  *total = s.i[nw - 1];
  __syncthreads();
  return before + x - flag;
}

// Exclusive scan like block_excl_scan with one barrier: the per-warp totals go to one of two
// buffers chosen by the caller's running call count `it`, so the next call (which writes the
// other buffer after its own barrier) cannot race with this call's reads.  Consecutive calls
// must pass consecutive `it` values.
DEV int block_scan_db(int flag, int* total, int (*buf)[33], int it) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = flag;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  int* b = buf[it & 1];
  if (lane == 31) b[wid] = x;
  __syncthreads();
  int before = 0, tot = 0;
  for (int w = 0; w < nw; ++w) {
    const int v = b[w];
    before += w < wid ? v : 0;
    tot += v;
  }
  *total = tot;
  return before + x - flag;
}

// order-preserving double <-> uint64 map (total order, -0.0 < +0.0)
DEV uint64_t d_ord(double v) {
  const uint64_t u = (uint64_t)__double_as_longlong(v);
  return (u >> 63) ? ~u : (u | 0x8000000000000000ull);
}
DEV double d_unord(uint64_t k) {
  const uint64_t u = (k >> 63) ? (k & 0x7fffffffffffffffull) : ~k;
  return __longlong_as_double((long long)u);
}

// Exact k-th smallest (0-based) of a[0..n) by MSB-first radix selection on the ordered bit
// pattern: returns exactly the value std::nth_element leaves at position k.
// hist: SEL_HIST(1) shared ints.  All threads of the block must call it.
DEV void block_select_multi(const double* const* a, const int* n, const int* kq, double* out, int nq, int* hist, BlockScratch& s,
                            unsigned long long* list = nullptr);
DEV double block_select(const double* a, int n, int k, int* hist, BlockScratch& s, unsigned long long* list = nullptr) {
  __shared__ double sel1;
  const double* arr[1] = {a};
  const int nn[1] = {n}, kk[1] = {k};
  block_select_multi(arr, nn, kk, &sel1, 1, hist, s, list);
  return sel1;
}

// Up to SEL_MAXQ exact selections at once: value q = the k[q]-th smallest of a[q][0..n[q]).
// Keys are the ordered bit patterns.  The bits every key of an array shares (its minimum and
// maximum agree on them) are decided first; then each query walks the remaining bits MSB first,
// 8 per round, with one histogram of the keys under its decided prefix per round.  Queries on
// the same array share the first histogram (their prefixes only part after it).  Once the
// chosen digit holds at most SEL_GATHER keys, those are gathered and ranked by one warp instead
// of running the remaining rounds.  With list (nq x SEL_LIST shared words), a query whose chosen
// digit holds at most SEL_LIST keys copies them to its list in the next round, and the rounds
// after that read only the list.  Two barriers per round.
// hist: SEL_HIST(nq) shared ints.  Needs nq <= warps of the block.  All threads must call it.
#define SEL_MAXQ 9
#define SEL_GATHER 32
#define SEL_LIST 256
#define SEL_HIST(nq) (2 * (nq) * 256)
DEV void block_select_multi(const double* const* a, const int* n, const int* kq, double* out, int nq, int* hist, BlockScratch& s,
                            unsigned long long* list) {
  __shared__ unsigned long long sh_prefix[SEL_MAXQ], sh_mn[SEL_MAXQ], sh_mx[SEL_MAXQ];
  __shared__ unsigned long long sh_g[SEL_MAXQ][SEL_GATHER];
  __shared__ int sh_k[SEL_MAXQ], sh_dec[SEL_MAXQ], sh_mode[SEL_MAXQ], sh_gn[SEL_MAXQ], sh_first[SEL_MAXQ], sh_ld[SEL_MAXQ], sh_live;
  __shared__ int sh_lst[SEL_MAXQ], sh_ln[SEL_MAXQ];   // list state (0 none, 1 filling this round, 2 filled), length
  const int tid = threadIdx.x, lane = tid & 31, wq = tid >> 5;
  int* hist0 = hist + nq * 256;   // first histogram of each group leader (queries on one array share it)
#ifdef SMG_CHECKS
  if (tid == 0 && (nq > SEL_MAXQ || nq > (int)(blockDim.x >> 5))) smg_chk_fail(132, nq, SEL_MAXQ);
  if (tid < nq && (kq[tid] < 0 || kq[tid] >= n[tid])) smg_chk_fail(130, kq[tid], n[tid]);
#endif
  for (int i = tid; i < 2 * nq * 256; i += blockDim.x) hist[i] = 0;
  if (tid < nq) {
    int ld = tid;
    for (int q = 0; q < tid; ++q)
      if (a[q] == a[tid] && n[q] == n[tid]) { ld = q; break; }
    sh_ld[tid] = ld;
    sh_k[tid] = kq[tid]; sh_mode[tid] = 0; sh_gn[tid] = 0; sh_first[tid] = 1; sh_mn[tid] = ~0ull; sh_mx[tid] = 0ull;
    sh_lst[tid] = 0; sh_ln[tid] = 0;
  }
  if (tid == 0) sh_live = nq;
  __syncthreads();
  // the bits every key of an array shares (its minimum and maximum agree on them) are decided first
  for (int q = 0; q < nq; ++q) {
    if (sh_ld[q] != q) continue;
    unsigned long long mn = ~0ull, mx = 0ull;
    for (int i = tid; i < n[q]; i += blockDim.x) {
      const unsigned long long key = d_ord(a[q][i]);
      mn = key < mn ? key : mn;
      mx = key > mx ? key : mx;
    }
    // warp min / max of the 64-bit keys as two 32-bit reductions (high word, then low word)
    const unsigned hmn = __reduce_min_sync(0xffffffffu, (unsigned)(mn >> 32));
    const unsigned lmn = __reduce_min_sync(0xffffffffu, (unsigned)(mn >> 32) == hmn ? (unsigned)mn : 0xffffffffu);
    const unsigned hmx = __reduce_max_sync(0xffffffffu, (unsigned)(mx >> 32));
    const unsigned lmx = __reduce_max_sync(0xffffffffu, (unsigned)(mx >> 32) == hmx ? (unsigned)mx : 0u);
    if (lane == 0) {
      atomicMin(&sh_mn[q], ((unsigned long long)hmn << 32) | lmn);
      atomicMax(&sh_mx[q], ((unsigned long long)hmx << 32) | lmx);
    }
  }
  __syncthreads();
  if (tid < nq) {
    const unsigned long long mn = sh_mn[sh_ld[tid]], d = mn ^ sh_mx[sh_ld[tid]];
    const int dec = d ? __clzll((long long)d) : 64;
    sh_dec[tid] = dec;
    sh_prefix[tid] = dec == 0 ? 0ull : mn & (~0ull << (64 - dec));
    if (dec == 64 || n[tid] <= 0) {   // all keys equal (or none)
      out[tid] = d_unord(mn);
      sh_mode[tid] = 2;
      atomicSub(&sh_live, 1);
    }
  }
  __syncthreads();
  for (int round = 0; round < 10; ++round) {
    // A: histogram (mode 0) or gather (mode 1) of the keys under each query's prefix; the first
    // histogram of a group is taken by its leader alone
    for (int q = 0; q < nq; ++q) {
      const int mode = sh_mode[q], first = sh_first[q];
      if (mode == 2 || (mode == 0 && first && sh_ld[q] != q)) continue;
      const int dec = sh_dec[q];
      const uint64_t pre = sh_prefix[q], msk = dec == 0 ? 0ull : ~0ull << (64 - dec);
      const int wdt = 64 - dec < 8 ? 64 - dec : 8, shift = 64 - dec - wdt;   // next digit: bits [shift, shift + wdt)
      int* hq = (first ? hist0 : hist) + q * 256;
      const int lst = sh_lst[q];
      unsigned long long* lq = list ? list + (size_t)q * SEL_LIST : nullptr;
      const double* aq = a[q];
      const int nqq = lst == 2 ? sh_ln[q] : n[q];
      for (int i = tid; i < nqq; i += blockDim.x) {
        const uint64_t key = lst == 2 ? lq[i] : d_ord(aq[i]);
        if ((key & msk) != pre) continue;
        if (lst == 1) {   // the keys under the new prefix go to the query's list
          const int slot = atomicAdd(&sh_ln[q], 1);
          if (INB(slot, SEL_LIST, 134)) lq[slot] = key;
        }
        if (mode == 0) {
          atomicAdd(&hq[(unsigned)(key >> shift) & ((1u << wdt) - 1u)], 1);
        } else {
          const int slot = atomicAdd(&sh_gn[q], 1);
          if (INB(slot, SEL_GATHER, 133)) sh_g[q][slot] = key;
        }
      }
    }
    __syncthreads();
    // B: warp q picks the digit holding rank k (clearing its own counters), or ranks the gathered keys
    if (wq < nq && sh_lst[wq] == 1) {   // the list was filled in this round's pass
      __syncwarp();
      if (lane == 0) sh_lst[wq] = 2;
      __syncwarp();
    }
    if (wq < nq && sh_mode[wq] != 2) {
      const int k = sh_k[wq];
      if (sh_mode[wq] == 0) {
        const int first = sh_first[wq];
        int* hq = first ? hist0 + sh_ld[wq] * 256 : hist + wq * 256;
        int c[8], tot = 0;
        for (int j = 0; j < 8; ++j) { c[j] = hq[lane * 8 + j]; tot += c[j]; }
        if (!first)
          for (int j = 0; j < 8; ++j) hq[lane * 8 + j] = 0;
        int incl = tot;
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const int excl = incl - tot;
        const int all = __shfl_sync(0xffffffffu, incl, 31);
        if (lane == 0) sh_first[wq] = 0;
        if (k >= excl && k < incl) {
          int kk = k - excl, b = 0;
          for (int j = 0; j < 8; ++j) {
            if (kk < c[j]) { b = j; break; }
            kk -= c[j];
          }
          const int d0 = sh_dec[wq], wdt = 64 - d0 < 8 ? 64 - d0 : 8, dec = d0 + wdt;
          sh_prefix[wq] |= (unsigned long long)(lane * 8 + b) << (64 - dec);
          sh_k[wq] = kk;
          sh_dec[wq] = dec;
          if (dec == 64) {
            out[wq] = d_unord(sh_prefix[wq]);
            sh_mode[wq] = 2;
            atomicSub(&sh_live, 1);
          } else if (c[b] <= SEL_GATHER) {
            sh_mode[wq] = 1;
          } else if (list && sh_lst[wq] == 0 && c[b] <= SEL_LIST) {
            sh_lst[wq] = 1;   // the next round copies the chosen digit's keys to the list
            sh_ln[wq] = 0;
          }
        } else if (lane == 0 && !(k >= 0 && k < all)) {   // rank outside the keys: no selection
          out[wq] = d_unord(sh_prefix[wq]);
          sh_mode[wq] = 2;
          atomicSub(&sh_live, 1);
        }
      } else {
        const int gn = sh_gn[wq] < SEL_GATHER ? sh_gn[wq] : SEL_GATHER;
        const uint64_t g = lane < gn ? sh_g[wq][lane] : 0ull;
        int lt = 0, eq = 0;
        for (int j = 0; j < gn; ++j) {
          const uint64_t h = sh_g[wq][j];
          lt += h < g;
          eq += h == g;
        }
        const bool hit = lane < gn && lt <= k && k < lt + eq;
        const unsigned hm = __ballot_sync(0xffffffffu, hit);
        if (lane == (hm ? __ffs(hm) - 1 : 0)) {
          out[wq] = d_unord(hm ? g : sh_prefix[wq]);
          sh_mode[wq] = 2;
          atomicSub(&sh_live, 1);
        }
      }
    }
    __syncthreads();
    PHASE_COUNT(40 + round);   // selection rounds (instrumentation builds)
    if (sh_live == 0) break;
  }
  (void)s;
}

// ---------------------------------------------------------------- hashing / keys
// splitmix64 step and seed mixing (scenemap objprob.cpp:116-128)
DEV uint64_t splitmix(uint64_t& s) {
  uint64_t z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
DEV uint64_t ap_seed(uint64_t a, uint64_t b) {
  uint64_t s = a * 0x9E3779B97F4A7C15ull ^ (b + 0x632BE59BD9B4E019ull);
  return splitmix(s);
}
// 21-bit packed voxel key of float coordinates (scenemap cloud.cpp:66-69)
DEV uint64_t voxel_key(float x, float y, float z, float inv) {
  const uint64_t qx = (uint64_t)((long long)floorf(x * inv) + (1 << 20)) & 0x1FFFFFull;
  const uint64_t qy = (uint64_t)((long long)floorf(y * inv) + (1 << 20)) & 0x1FFFFFull;
  const uint64_t qz = (uint64_t)((long long)floorf(z * inv) + (1 << 20)) & 0x1FFFFFull;
  return qx | qy << 21 | qz << 42;
}
// 21-bit packed contact-cell key (scenemap objprob.cpp:92-95)
DEV uint64_t cell_key3(long long i, long long j, long long k) {
  return ((uint64_t)(i + (1 << 20)) & 0x1FFFFFull) | ((uint64_t)(j + (1 << 20)) & 0x1FFFFFull) << 21 |
         ((uint64_t)(k + (1 << 20)) & 0x1FFFFFull) << 42;
}
// 64-bit mixer for open addressing (device-side tables only; not a reference structure)
DEV uint32_t hmix(uint64_t k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return (uint32_t)k;
}

// float -> fp16 bits with the reference's own rounding (scenemap objprob.cpp:12-29): round half
// up on the mantissa, small numbers flushed per its subnormal rule.  Integer-only, bit-exact.
DEV uint16_t ref_f2h(float f) {
  const uint32_t x = __float_as_uint(f);
  const uint32_t sign = (x >> 16) & 0x8000u;
  int32_t e = (int32_t)((x >> 23) & 0xff) - 127 + 15;
  uint32_t m = x & 0x7fffffu;
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    m |= 0x800000u;
    const int sh = 14 - e;
    return (uint16_t)(sign | ((m + (1u << (sh - 1))) >> sh));
  }
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  const uint32_t r = m + 0x1000u;
  if (r & 0x800000u) {
    m = 0;
    ++e;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  } else {
    m = r;
  }
  return (uint16_t)(sign | ((uint32_t)e << 10) | (m >> 13));
}
// fp16 bits -> float (scenemap objprob.cpp:31-47; exact widening)
// fp16 -> fp32 is exact for every finite value and infinity (what the reference's bitwise
// widening computes); the hardware conversion gives the same floats, NaN stays NaN.
DEV float ref_h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

DEV float emb_at(const void* emb, int dtype, int D, int k, int i) {
  if (dtype == SMG_EMB_BF16) {
    const uint16_t b = ((const uint16_t*)emb)[(size_t)k * D + i];
    return __uint_as_float((uint32_t)b << 16);
  }
  return ((const float*)emb)[(size_t)k * D + i];
}

// ---------------------------------------------------------------- objprob scalar math
// (scenemap include/scenemap/objprob_math.h, T = double)
// opm::max2/min2/max3 (objprob_math.h:16-18)
DEV double dmax2(double a, double b) { return a > b ? a : b; }
DEV double dmin2(double a, double b) { return a < b ? a : b; }
DEV double dmax3(double a, double b, double c) { return dmax2(dmax2(a, b), c); }
// std::max / std::min (returns the first argument on ties, like <algorithm>)
DEV double smax(double a, double b) { return (a < b) ? b : a; }
DEV double smin(double a, double b) { return (b < a) ? b : a; }
// std::max({0.0, a, b}) (first largest of an initializer list)
DEV double smax3(double a, double b, double c) { double r = a; if (r < b) r = b; if (r < c) r = c; return r; }

// objprob_math.h:25-30
DEV double same_logit(const double w[8], const double f[7]) {
  double v = w[0];
  for (int k = 0; k < 7; ++k) v += w[k + 1] * f[k];
  if (f[5] > 0) v = -30.0;
  return v;
}
DEV double sigmoid(double x) { return 1.0 / (1.0 + exp(-x)); }

// objprob_math.h:34-45 (da boxOverlap, da/src/merge.cpp:8-20)
DEV double box_overlap(const double alo[3], const double ahi[3], const double blo[3], const double bhi[3], double min_ext) {
  double r = 1.0;
  for (int k = 0; k < 3; ++k) {
    const double ca = 0.5 * (alo[k] + ahi[k]), cb = 0.5 * (blo[k] + bhi[k]);
    const double ha = 0.5 * dmax2(ahi[k] - alo[k], min_ext), hb = 0.5 * dmax2(bhi[k] - blo[k], min_ext);
    const double ov = dmin2(ca + ha, cb + hb) - dmax2(ca - ha, cb - hb);
    const double f = ov <= 0 ? 0.0 : dmin2(1.0, ov / (2.0 * dmin2(ha, hb)));
    r *= f;
    if (r <= 0) return 0.0;
  }
  return r;
}

// objprob_math.h:49-74
DEV void pair_geo(const double alo[3], const double ahi[3], const double apos[3], const double blo[3], const double bhi[3],
                  const double bpos[3], double cs, double cos0, double f[7]) {
  double g2 = 0;
  for (int k = 0; k < 3; ++k) {
    const double g = dmax3(0.0, alo[k] - bhi[k], blo[k] - ahi[k]);
    g2 += g * g;
  }
  f[1] = sqrt(g2);
  const double ea = dmax3(ahi[0] - alo[0], ahi[1] - alo[1], ahi[2] - alo[2]);
  const double eb = dmax3(bhi[0] - blo[0], bhi[1] - blo[1], bhi[2] - blo[2]);
  const double dd = sqrt((apos[0] - bpos[0]) * (apos[0] - bpos[0]) + (apos[1] - bpos[1]) * (apos[1] - bpos[1]) +
                         (apos[2] - bpos[2]) * (apos[2] - bpos[2]));
  f[2] = dd / (0.5 * (ea + eb) + 0.05);
  f[3] = cs > -1.5 ? cs - cos0 : 0.0;
  f[4] = box_overlap(alo, ahi, blo, bhi, 0.05);
  const bool a_small = ea < eb;
  const double *slo = a_small ? alo : blo, *shi = a_small ? ahi : bhi, *llo = a_small ? blo : alo, *lhi = a_small ? bhi : ahi;
  const double es = dmin2(ea, eb), el = dmax2(ea, eb);
  f[5] = 0.0;
  if (es < 0.6 * el) {
    const double cx = 0.5 * (slo[0] + shi[0]), cy = 0.5 * (slo[1] + shi[1]);
    const bool inside = cx > llo[0] - 0.05 && cx < lhi[0] + 0.05 && cy > llo[1] - 0.05 && cy < lhi[1] + 0.05;
    const double dz = slo[2] - lhi[2];
    if (inside && (dz < 0 ? -dz : dz) < 0.08) f[5] = 1.0;
  }
}

// objprob_math.h:78-87 with occ/blur handled by the caller-provided factors
DEV double view_kappa(double size_px, bool trunc, double depth, double k0, double s0, double trunc_k, double d0, double occ,
                      double blur_w, double blur_fac) {
  const double s = dmax2(0.0, size_px), d = dmax2(0.0, depth);
  double k = k0 * s / (s + s0);
  if (trunc) k *= trunc_k;
  k /= 1.0 + (d / d0) * (d / d0);
  k *= pow(1.0, occ);   // vis = 1 for detection fragments: pow(1, y) == 1 exactly
  if (blur_w > 0) k *= blur_fac;
  return dmax2(k, 1e-3);
}

// objprob_math.h:139-156
DEV double kalman_gain(double& P, double q, double dt, double R) {
  P += q * dmax2(0.0, dt);
  const double K = P / (P + R);
  P *= 1.0 - K;
  return K;
}
DEV double kalman_R(double r0, double r1, double depth, bool trunc, double ext) {
  const double sd = r0 + r1 * depth;
  return sd * sd + (trunc ? 0.25 * ext * ext : 0.0);
}
DEV void kalman_big(double& P, double q, double dt, double sd, double ext) {
  const double R = sd * sd + 0.0625 * ext * ext;
  P = 1.0 / (1.0 / (P + q * dmax2(0.0, dt)) + 1.0 / R);
}
DEV double merge_var(double a, double b) { return 1.0 / (1.0 / dmax2(a, 1e-9) + 1.0 / dmax2(b, 1e-9)); }

// 3-argument hypot by scaling with the largest magnitude
DEV double hypot3(double x, double y, double z) {
  x = fabs(x); y = fabs(y); z = fabs(z);
  const double a = dmax3(x, y, z);
  if (a == 0.0) return 0.0;
  x /= a; y /= a; z /= a;
  return a * sqrt(x * x + y * y + z * z);
}
// segDist (scenemap objmap.cpp:77-84): horizontal distance from (px, py) to segment s = (ax, ay,
// bx, by), the parameter clamped to [0, 1]
DEV double seg_dist(double px, double py, const double* s) {
  const double ax = s[0], ay = s[1], bx = s[2], by = s[3];
  const double dx = bx - ax, dy = by - ay, l2 = dx * dx + dy * dy;
  double u = l2 > 1e-12 ? ((px - ax) * dx + (py - ay) * dy) / l2 : 0.0;
  u = u < 0.0 ? 0.0 : (1.0 < u ? 1.0 : u);
  return hypot(px - ax - u * dx, py - ay - u * dy);
}
// min over the first segments of the set until one lies within `stop` (the reference's early-out
// loops): the result is <= stop exactly when some segment does
DEV double wall_dist(double px, double py, const double* S, int n, double stop) {
  double dm = 1e9;
  for (int k = 0; k < n && dm > stop; ++k) dm = smin(dm, seg_dist(px, py, S + 4 * k));
  return dm;
}
DEV double dist3(const double* a, const double* b) {
  return sqrt((a[0] - b[0]) * (a[0] - b[0]) + (a[1] - b[1]) * (a[1] - b[1]) + (a[2] - b[2]) * (a[2] - b[2]));
}

DEV void set_err(MapRec* m, int bit) { atomicOr(&m->err, bit); }


// global index of cloud slot `slot` of map m (clouds are a pool of B.C slots per map, separate
// from the B.O object slots)
__host__ __device__ inline size_t cglob(const Batch& B, int m, int slot) { return (size_t)m * B.C + slot; }

// Scan box of detection k in depth pixels (objmap.cpp:648-652): the detector box scaled from
// the detector image to the depth image (float scale, truncation to int), grown by one pixel
// and clipped to the frame.
DEV void det_scan_box(const FrameDev& F, int k, int* u0, int* u1, int* v0, int* v1) {
  const float* b = F.box[k];
  *u0 = max(0, (int)(b[0] * F.sxu_f) - 1);
  *u1 = min(F.w - 1, (int)(b[2] * F.sxu_f) + 1);
  *v0 = max(0, (int)(b[1] * F.syv_f) - 1);
  *v1 = min(F.h - 1, (int)(b[3] * F.syv_f) + 1);
}

// Bit-mask form of detection k's mask (sm_detections): depth pixel (u, v) -> detector pixel
// centre -> mask cell, 1-cell 4-neighbour erosion, rows at the grid's edge skipped
// (objmap.cpp:655-678).  pu, pv: the detector pixel (PU, PV of the observation's points).
DEV bool det_bits_at(const FrameDev& F, int k, int u, int v, int* pu, int* pv) {
  const float yi = ((float)v + 0.5f) / F.syv_f;
  const int j = (int)floorf((yi - F.mask_oy) / F.mask_sy);
  const int MW = F.mask_w, MH = F.mask_h;
  if (j < 1 || j >= MH - 1) return false;
  const float xi = ((float)u + 0.5f) / F.sxu_f;
  const int i = (int)floorf((xi - F.mask_ox) / F.mask_sx);
  const uint32_t* bits = F.mask_bits + (size_t)k * F.mask_words;
  auto bit = [&](int a, int c) -> bool {
    if (a < 0 || c < 0 || a >= MW || c >= MH) return false;
    const size_t q = (size_t)c * MW + a;
    return (bits[q >> 5] >> (q & 31)) & 1u;
  };
  *pu = (int)xi;
  *pv = (int)yi;
  return bit(i, j) && bit(i - 1, j) && bit(i + 1, j) && bit(i, j - 1) && bit(i, j + 1);
}
DEV void wk_add(MapRec* m, int k, long long v) {
  if (v) atomicAdd((unsigned long long*)&m->wk[k], (unsigned long long)v);
}

// event in program order: key = phase << 24 | position
// camera ring of an object (the newest SMG_CAMS cameras, oldest first): entry i, and an append
// that drops the oldest when full (push, then erase the front)
DEV double* cam_at(ObjRec& o, int i) { return o.cams[(o.cam_head + i) & (SMG_CAMS - 1)]; }
DEV const double* cam_at(const ObjRec& o, int i) { return o.cams[(o.cam_head + i) & (SMG_CAMS - 1)]; }
DEV void cam_push(ObjRec& o, const double c[7]) {
  double* d;
  if (o.n_cams >= SMG_CAMS) {
    d = o.cams[o.cam_head & (SMG_CAMS - 1)];
    o.cam_head = (o.cam_head + 1) & (SMG_CAMS - 1);
    o.n_cams = SMG_CAMS;
  } else {
    d = cam_at(o, o.n_cams++);
  }
  for (int j = 0; j < 7; ++j) d[j] = c[j];
}

DEV void push_event(const Batch& B, int map, double t, const ObjRec& o, int kind, uint32_t key) {
  MapRec* M = &B.maps[map];
  const int e = atomicAdd(&M->n_events, 1);
  if (e >= SMG_MAX_EVENTS) { set_err(M, SMG_E_CAP_EVENTS); return; }
  EventRec& r = B.events[(size_t)map * SMG_MAX_EVENTS + e];
  r.t = t;
  r.id = o.id;
  r.kind = kind;
  r.key = key;
}

// ---------------------------------------------------------------- class kinds and names
DEV int kind_of(const Batch& B, int cls) {   // ObjectMap::kindOf (objmap.hpp:246)
  return B.txt.kinds && cls >= 0 && cls < B.txt.n_labels ? (int)B.txt.kinds[cls] : KIND_OBJECT;
}
// ObjectMap::exportable (objmap.hpp:273-279) with export_named on (the only setting accepted
// here): confirmed, named (a posterior), not hidden, not the fallback name, not a structure label
DEV bool exportable(const Batch& B, const ObjRec& o) {
  if (!o.confirmed || !o.has_post || o.hide) return false;
  if (B.txt.object_label >= 0 && o.cls == B.txt.object_label) return false;
  return kind_of(B, o.cls) != KIND_STRUCTURE;
}
// ObjectMap::isBig (objmap.cpp:207-209)
DEV bool is_big(const Batch& B, const ObjRec& o) {
  const int k = kind_of(B, o.cls);
  return k == KIND_STATIC || k == KIND_STRUCT_OBJ || smax(smax(o.hi[0] - o.lo[0], o.hi[1] - o.lo[1]), o.hi[2] - o.lo[2]) > B.p.big;
}
// flatNamed (objmap.hpp:306-308): the object's name is a wall-mounted flat object
DEV bool flat_named(const Batch& B, const ObjRec& o) {
  return B.txt.flat_ok && o.name_lab >= 0 && o.name_lab < B.txt.n_labels && B.txt.flat_ok[o.name_lab];
}
// ObjectMap::labelRelated (objmap.cpp:1243-1253): equal, or one an ancestor of the other
DEV bool label_related(const Batch& B, int a, int b) {
  if (a == b) return true;
  const int* par = B.txt.parent;
  const int C = B.txt.n_labels;
  auto up = [&](int x, int y) {
    for (int g = 0; x >= 0 && g < 8; ++g) {
      x = par && x < C ? par[x] : -1;
      if (x == y) return true;
    }
    return false;
  };
  return up(a, b) || up(b, a);
}
