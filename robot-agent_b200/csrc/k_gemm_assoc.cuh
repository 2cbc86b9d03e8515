// Association stress path: detections x memory bank on the tcgen05 tensor
// cores, with the association decision fused into the epilogue.
//
// Score of (detection d, memory j) = dot(z_d, m_j) of the bf16 L2-normalised embeddings, fp32
// accumulation in TMEM.  A pair takes part only if the 3D boxes overlap with IoU > iou_min
// (float arithmetic, the same operation order as the CPU restatement).  Decision per
// detection: the gated memory with the largest score if that score is >= cos_min, the lowest
// memory index on ties, else no match -- evaluated on the fp64 dot products of the same bf16
// values summed in index order (the restatement's definition).
//
// The tensor-core scores differ from those fp64 values by at most `delta` (fp32 accumulation
// of K exact bf16 products of unit vectors: K * 2^-23 bounds it; the host passes a margin
// above that).  The epilogue keeps, per detection and tile, the best and second-best gated
// scores; k_assoc_decide certifies a decision when the best is clear of the threshold and of
// the runner-up by more than the error margin, and otherwise recomputes that detection's gated
// candidates in fp64, in index order, so every decision equals the restatement's.
//
// GEMM: A = detections [n_det][K], B = memories [n_mem][K], both K-major bf16, loaded by TMA
// (128-byte swizzle, 64-element K blocks) into a 4-stage shared-memory ring; one elected
// thread issues tcgen05.mma (M = 128, N = 256, K = 16) into a 128 x 256 fp32 TMEM
// accumulator; the four warps read it back with tcgen05.ld (warp w owns TMEM lanes 32w..32w+31,
// i.e. detections), apply the gate and keep the top-2 per detection.  Every mbarrier wait is
// bounded by a %globaltimer limit; a timeout sets the error word and the CTA still waits
// (bounded) for its tensor-core work and frees its TMEM before returning.
#pragma once
#include <cuda.h>
#include "dev_util.cuh"

#define AG_BM 128
#define AG_BN 256
#define AG_BK 64
#define AG_STAGES 4
#define AG_THREADS 512   // 16 warps: warps w, w+4, w+8, w+12 read the same TMEM lanes, a quarter of the columns each
#define AG_GROUPS (AG_THREADS / 128)
#define AG_A_BYTES (AG_BM * AG_BK * 2)
#define AG_B_BYTES (AG_BN * AG_BK * 2)
#define AG_TMEM_COLS 256
#define AG_SMEM (AG_STAGES * (AG_A_BYTES + AG_B_BYTES) + 1024 + 256 + AG_BN * 8 * 4 + AG_GROUPS * AG_BM * 3 * 4)
#define AG_WAIT_NS 200000000ull   // 0.2 s per wait

// instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A bf16 (bits 7-9 = 1), B bf16
// (bits 10-12 = 1), both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28
#define AG_IDESC ((1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(AG_BN >> 3) << 17) | ((uint32_t)(AG_BM >> 4) << 24))

struct AssocArgs {
  int n_det, n_mem, dim, n_tiles;
  const float* det_box;   // n_det x 6: lo xyz, hi xyz
  const float* mem_box;   // n_mem x 6
  const uint16_t* det;    // n_det x dim bf16
  const uint16_t* mem;    // n_mem x dim bf16
  float iou_min;
  double cos_min, delta;
  float* t_best;          // [n_det][n_tiles]
  float* t_second;
  int32_t* t_idx;
  float* scores;          // optional [n_det][n_mem]
  int32_t* match;         // [n_det]
  double* score;          // [n_det]
  int32_t* certified;     // [n_det] 1 = decided from the tensor-core scores, 0 = recomputed
  int32_t* err;           // [1]
  unsigned long long* stamps;   // optional: %globaltimer at 16 points of CTA (0, 0) (instrumentation)
};

DEV uint32_t ag_smem(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

DEV uint64_t ag_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

DEV void ag_mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(ag_smem(b)), "r"(count) : "memory");
}

DEV void ag_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(ag_smem(b)), "r"(bytes) : "memory");
}

DEV bool ag_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(ag_smem(b)), "r"(parity)
      : "memory");
  return ok != 0;
}

// bounded wait on phase `parity`; false after AG_WAIT_NS
DEV bool ag_wait(uint64_t* b, uint32_t parity) {
  const uint64_t t0 = ag_now();
  for (uint32_t i = 0;; ++i) {
    if (ag_try_wait(b, parity)) return true;
    if ((i & 255u) == 255u && ag_now() - t0 > AG_WAIT_NS) return false;
  }
}

DEV void ag_tma_2d(const CUtensorMap* map, uint64_t* bar, void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          ag_smem(dst)),
      "l"((uint64_t)map), "r"(ag_smem(bar)), "r"(x), "r"(y)
      : "memory");
}

// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms 1024 bytes apart
DEV uint64_t ag_desc(const void* tile) {
  const uint32_t a = ag_smem(tile);
  uint64_t d = (uint64_t)((a >> 4) & 0x3fffu);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset
  d |= (uint64_t)1 << 46;             // descriptor version for tcgen05
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

DEV void ag_mma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem),
      "l"(da), "l"(db), "r"(AG_IDESC), "r"(accum));
}

DEV void ag_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(ag_smem(bar)) : "memory");
}

DEV void ag_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
DEV void ag_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

DEV void ag_tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

DEV void ag_tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 3D AABB IoU > tmin, float, fixed operation order (the restatement uses the same)
DEV bool ag_gate(const float* a, float avol, const float* b, float tmin) {
  float inter = 1.f;
  for (int k = 0; k < 3; ++k) {
    const float lo = fmaxf(a[k], b[k]), hi = fminf(a[3 + k], b[3 + k]);
    const float e = hi - lo;
    if (!(e > 0.f)) return false;
    inter = inter * e;
  }
  const float bvol = ((b[3] - b[0]) * (b[4] - b[1])) * (b[5] - b[2]);
  const float uni = (avol + bvol) - inter;
  return inter > tmin * uni;
}

__global__ void __launch_bounds__(AG_THREADS, 1)
    k_assoc_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, AssocArgs g) {
  extern __shared__ unsigned char ag_raw[];
  unsigned char* base = (unsigned char*)(((uintptr_t)ag_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* sA = base;
  unsigned char* sB = base + AG_STAGES * AG_A_BYTES;
  uint64_t* full = (uint64_t*)(sB + AG_STAGES * AG_B_BYTES);
  uint64_t* empty = full + AG_STAGES;
  uint64_t* done = empty + AG_STAGES;
  uint32_t* tmem_slot = (uint32_t*)(done + 1);
  float* mbox = (float*)(base + AG_STAGES * (AG_A_BYTES + AG_B_BYTES) + 256);
  __shared__ int sh_fail;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * AG_BN, m0 = blockIdx.y * AG_BM;
  const int nk = g.dim / AG_BK;
  const bool stamp = g.stamps && blockIdx.x == 0 && blockIdx.y == 0;
  if (stamp && tid == 0) g.stamps[0] = ag_now();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (tid == 0) {   // barriers, then the first AG_STAGES loads go out before anything else
    for (int s = 0; s < AG_STAGES; ++s) {
      ag_mbar_init(&full[s], 1);
      ag_mbar_init(&empty[s], 1);
    }
    ag_mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    sh_fail = 0;
    for (int kb = 0; kb < AG_STAGES && kb < nk; ++kb) {
      ag_expect_tx(&full[kb], AG_A_BYTES + AG_B_BYTES);
      ag_tma_2d(&tmA, &full[kb], sA + kb * AG_A_BYTES, kb * AG_BK, m0);
      ag_tma_2d(&tmB, &full[kb], sB + kb * AG_B_BYTES, kb * AG_BK, n0);
    }
    if (stamp) g.stamps[2] = ag_now();
  }
  // memory boxes of the tile: lo xyz, hi xyz, volume ((dx * dy) * dz), pad
  for (int c = tid; c < AG_BN; c += blockDim.x) {
    const int j = n0 + c;
    float b[6] = {0, 0, 0, 0, 0, 0};
    if (j < g.n_mem)
      for (int k = 0; k < 6; ++k) b[k] = g.mem_box[(size_t)j * 6 + k];
    float* o = mbox + 8 * c;
    for (int k = 0; k < 6; ++k) o[k] = b[k];
    o[6] = ((b[3] - b[0]) * (b[4] - b[1])) * (b[5] - b[2]);
    o[7] = 0.f;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(ag_smem(tmem_slot)),
                 "r"(AG_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  ag_fence_before();
  __syncthreads();
  ag_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (stamp && tid == 0) g.stamps[1] = ag_now();

  if (warp == 0 && lane == 0) {   // TMA producer (the first AG_STAGES loads are already out)
    for (int kb = AG_STAGES; kb < nk; ++kb) {
      const int s = kb % AG_STAGES;
      const uint32_t ph = (uint32_t)(kb / AG_STAGES) & 1u;
      if (!ag_wait(&empty[s], ph ^ 1u)) { sh_fail = 1; break; }
      ag_expect_tx(&full[s], AG_A_BYTES + AG_B_BYTES);
      ag_tma_2d(&tmA, &full[s], sA + s * AG_A_BYTES, kb * AG_BK, m0);
      ag_tma_2d(&tmB, &full[s], sB + s * AG_B_BYTES, kb * AG_BK, n0);
    }
  } else if (warp == 1 && lane == 0) {   // MMA issuer
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % AG_STAGES;
      const uint32_t ph = (uint32_t)(kb / AG_STAGES) & 1u;
      if (!ag_wait(&full[s], ph)) { sh_fail = 1; break; }
      if (stamp && kb == 0) g.stamps[3] = ag_now();
      if (stamp && kb == nk - 1) g.stamps[4] = ag_now();
      ag_fence_after();
      const uint64_t da = ag_desc(sA + s * AG_A_BYTES), db = ag_desc(sB + s * AG_B_BYTES);
#pragma unroll
      for (int k = 0; k < AG_BK / 16; ++k) ag_mma(tmem, da + 2 * k, db + 2 * k, (kb | k) != 0);
      ag_commit(&empty[s]);
    }
    ag_commit(done);   // also on failure: arrives once every issued MMA has completed
  }
  __syncwarp();
  bool ok = ag_wait(done, 0);
  if (warp == 0 && lane == 0) {   // drain: the last loads issued must have landed before exit
    for (int kb = nk - AG_STAGES > 0 ? nk - AG_STAGES : 0; kb < nk; ++kb)
      ok = ag_wait(&full[kb % AG_STAGES], (uint32_t)(kb / AG_STAGES) & 1u) && ok;
  }
  ok = __syncthreads_and(ok ? 1 : 0) != 0;
  if (stamp && tid == 0) g.stamps[5] = ag_now();
  ag_fence_after();
  const int quarter = warp & 3, grp = warp >> 2;   // TMEM lane quarter, column group
  const int r = quarter * 32 + lane, d = m0 + r;
  float bx[6] = {0, 0, 0, 0, 0, 0};
  if (d < g.n_det)
    for (int k = 0; k < 6; ++k) bx[k] = g.det_box[(size_t)d * 6 + k];
  const float avol = ((bx[3] - bx[0]) * (bx[4] - bx[1])) * (bx[5] - bx[2]);
  if (stamp && tid == 0) g.stamps[8] = ag_now();
  const float tmin = g.iou_min;
  const float4* mb4 = (const float4*)mbox;
  float b1 = -INFINITY, b2 = -INFINITY;
  int i1 = -1;
  const int jlim = g.n_mem - n0;   // columns c < jlim are real memories
  constexpr int CW = AG_BN / AG_GROUPS;
  if (ok) {
    for (int c0 = grp * CW; c0 < (grp + 1) * CW; c0 += 16) {
      uint32_t v[16];
      ag_tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0, v);
      if (stamp && tid == 0 && c0 == 0) g.stamps[9] = ag_now();
      if (g.scores && d < g.n_det) {
#pragma unroll
        for (int c = 0; c < 16; ++c)
          if (c0 + c < jlim) g.scores[(size_t)d * g.n_mem + n0 + c0 + c] = __uint_as_float(v[c]);
      }
      // pass 1: x and y overlap (a superset of the gate), one bit per column; the warp's OR
      uint32_t mine = 0;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float4 p = mb4[2 * (c0 + c)], q = mb4[2 * (c0 + c) + 1];   // lo xyz hi.x | hi.y hi.z vol pad
        const float e0 = fminf(bx[3], p.w) - fmaxf(bx[0], p.x);
        const float e1 = fminf(bx[4], q.x) - fmaxf(bx[1], p.y);
        mine |= (uint32_t)(e0 > 0.f && e1 > 0.f && c0 + c < jlim) << c;
      }
      const uint32_t any = __reduce_or_sync(0xffffffffu, mine);
      if (!any) continue;
      // pass 2: the full gate (the same float operations as ag_gate and the restatement) and the
      // top-2 update, only on columns some lane of the warp still has; columns in increasing
      // order, so the first maximum keeps the lowest index
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        if (!((any >> c) & 1u)) continue;
        const float4 p = mb4[2 * (c0 + c)], q = mb4[2 * (c0 + c) + 1];
        const float e0 = fminf(bx[3], p.w) - fmaxf(bx[0], p.x);
        const float e1 = fminf(bx[4], q.x) - fmaxf(bx[1], p.y);
        const float e2 = fminf(bx[5], q.y) - fmaxf(bx[2], p.z);
        const float inter = (e0 * e1) * e2;
        const float uni = (avol + q.z) - inter;
        const bool pass = ((mine >> c) & 1u) && e2 > 0.f && inter > tmin * uni;
        const float sc = pass ? __uint_as_float(v[c]) : -INFINITY;
        const bool gt = sc > b1;
        b2 = gt ? b1 : fmaxf(b2, sc);
        i1 = gt ? n0 + c0 + c : i1;
        b1 = gt ? sc : b1;
      }
    }
  }
  if (stamp && tid == 0) g.stamps[10] = ag_now();
  // merge the column groups of each row in column order (ties keep the lower index)
  float* xb = (float*)(mbox + 8 * AG_BN);   // groups x 128 rows x (b1, b2, i1)
  if (grp > 0) {
    float* o = xb + 3 * ((size_t)grp * AG_BM + r);
    o[0] = b1;
    o[1] = b2;
    ((int*)o)[2] = i1;
  }
  __syncthreads();
  if (stamp && tid == 0) g.stamps[11] = ag_now();
  if (grp == 0) {
    for (int q2 = 1; q2 < AG_GROUPS; ++q2) {
      const float* o = xb + 3 * ((size_t)q2 * AG_BM + r);
      const float c1 = o[0], c2 = o[1];
      const int ci = ((const int*)o)[2];
      if (ci >= 0 && c1 > b1) { b2 = fmaxf(b1, c2); b1 = c1; i1 = ci; }
      else b2 = fmaxf(b2, c1);
    }
    if (d < g.n_det) {
      const size_t t = (size_t)d * g.n_tiles + blockIdx.x;
      g.t_best[t] = i1 >= 0 ? b1 : -INFINITY;
      g.t_second[t] = b2;
      g.t_idx[t] = i1;
    }
  }
  if (stamp && tid == 0) g.stamps[6] = ag_now();
  ag_fence_before();
  __syncthreads();
  if (tid == 0 && (sh_fail || !ok)) atomicOr(g.err, 1);
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(AG_TMEM_COLS) : "memory");
  }
  if (stamp && tid == 0) g.stamps[7] = ag_now();
}

// fp64 dot of two bf16 rows summed in index order (the restatement's definition)
DEV double ag_dot_seq(const uint16_t* a, const uint16_t* b, int D) {
  double s = 0.0;
  for (int k = 0; k < D; ++k) s += (double)__uint_as_float((uint32_t)a[k] << 16) * (double)__uint_as_float((uint32_t)b[k] << 16);
  return s;
}

// one warp per detection: combine the tiles, certify, or recompute in fp64
__global__ void __launch_bounds__(256) k_assoc_decide(AssocArgs g) {
  asm volatile("griddepcontrol.wait;" ::: "memory");   // the GEMM grid has completed (launched with PDL)
  const int lane = threadIdx.x & 31;
  const int d = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (d >= g.n_det) return;
  float b1 = -INFINITY, o1 = -INFINITY;   // best, and the best of the other candidates
  int i1 = 0x7fffffff;
  for (int t = lane; t < g.n_tiles; t += 32) {
    const size_t q = (size_t)d * g.n_tiles + t;
    const float tb = g.t_best[q], ts = g.t_second[q];
    const int ti = g.t_idx[q];
    if (ti >= 0 && (tb > b1 || (tb == b1 && ti < i1))) {
      o1 = fmaxf(o1, fmaxf(b1, ts));
      b1 = tb;
      i1 = ti;
    } else {
      o1 = fmaxf(o1, fmaxf(tb, ts));
    }
  }
  for (int off = 16; off > 0; off >>= 1) {
    const float b2 = __shfl_xor_sync(0xffffffffu, b1, off), p2 = __shfl_xor_sync(0xffffffffu, o1, off);
    const int j2 = __shfl_xor_sync(0xffffffffu, i1, off);
    if (j2 != 0x7fffffff && (b2 > b1 || (b2 == b1 && j2 < i1))) {
      o1 = fmaxf(p2, fmaxf(o1, b1));
      b1 = b2;
      i1 = j2;
    } else {
      o1 = fmaxf(o1, fmaxf(p2, b2));
    }
  }
  const double best = (double)b1, other = (double)o1, thr = g.cos_min, dl = g.delta;
  int decided = -2;   // -2 = undecided
  if (i1 == 0x7fffffff || best < thr - dl) decided = -1;
  else if (best >= thr + dl && other < best - 2 * dl) decided = i1;
  if (decided != -2) {
    double s = 0.0;
    if (decided >= 0) {   // fp64 score of the chosen pair (lane-parallel partial sums)
      // 16-byte loads (8 values), all of a lane's issued before its sums (rows are 16-byte
      // aligned: dim is a multiple of 64)
      const uint4* a = (const uint4*)(g.det + (size_t)d * g.dim);
      const uint4* b = (const uint4*)(g.mem + (size_t)decided * g.dim);
      const int n8 = g.dim >> 3;
#pragma unroll 4
      for (int q = lane; q < n8; q += 32) {
        const uint4 x = a[q], y = b[q];
        const uint32_t xa[4] = {x.x, x.y, x.z, x.w}, ya[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          s += (double)__uint_as_float(xa[e] << 16) * (double)__uint_as_float(ya[e] << 16);
          s += (double)__uint_as_float(xa[e] & 0xffff0000u) * (double)__uint_as_float(ya[e] & 0xffff0000u);
        }
      }
      s = warp_sum_d(s);
    }
    if (lane == 0) { g.match[d] = decided; g.score[d] = s; g.certified[d] = 1; }
    return;
  }
  // recompute: every gated memory, fp64 in index order, one lane per candidate
  float bx[6];
  for (int k = 0; k < 6; ++k) bx[k] = g.det_box[(size_t)d * 6 + k];
  const float avol = ((bx[3] - bx[0]) * (bx[4] - bx[1])) * (bx[5] - bx[2]);
  double bs = -1e300;
  int bj = 0x7fffffff;
  const uint16_t* a = g.det + (size_t)d * g.dim;
  for (int j = lane; j < g.n_mem; j += 32) {
    if (!ag_gate(bx, avol, g.mem_box + (size_t)j * 6, g.iou_min)) continue;
    const double s = ag_dot_seq(a, g.mem + (size_t)j * g.dim, g.dim);
    if (s >= thr && (s > bs || (s == bs && j < bj))) { bs = s; bj = j; }
  }
  for (int off = 16; off > 0; off >>= 1) {
    const double s2 = __shfl_xor_sync(0xffffffffu, bs, off);
    const int j2 = __shfl_xor_sync(0xffffffffu, bj, off);
    if (s2 > bs || (s2 == bs && j2 < bj)) { bs = s2; bj = j2; }
  }
  if (lane == 0) {
    g.match[d] = bj == 0x7fffffff ? -1 : bj;
    g.score[d] = bj == 0x7fffffff ? 0.0 : bs;
    g.certified[d] = 0;
  }
}

// ---- persistent form: many frames against one bank, epilogue overlapped with the next MMAs ----
//
// The frames of a batch are rows of one detection matrix (frame f's detections are rows
// f * n_det ..), so the batch is one GEMM of (frames x n_det) x n_mem x dim.  One CTA per SM walks
// the 128 x 256 tiles in column-major tile order (consecutive tiles share a bank tile, which the
// SMs running at the same time then read from L2 together).  Warp roles:
//   warp 0     TMA producer: A and B K-blocks into a 4-stage ring (full / empty mbarriers);
//   warp 1     MMA issuer: one elected thread, 72 tcgen05.mma per tile into one of two 256-column
//              TMEM accumulators (tfull[a] committed when a tile's MMAs have completed; it waits
//              on tempty[a] before reusing an accumulator);
//   warp 2     allocates and frees the 512 TMEM columns;
//   warps 4-11 epilogue: warp 4 + q + 4 h reads TMEM lanes 32q.. (detections) and columns
//              128h.. of the tile (memories), applies the gate, keeps the per-row best and
//              second-best, and writes them as tile-half 2 * (column tile) + h for k_assoc_decide;
//              then it arrives on tempty[a], so the MMAs of tile i + 2 can start while it works on
//              tile i + 1.
// Every wait is bounded (AG_WAIT_NS); a timeout sets the error word, the roles run out, and the
// CTA waits (bounded) for its issued loads and MMAs before freeing TMEM.
#define AP_EPI_WARPS 8
#define AP_THREADS ((4 + AP_EPI_WARPS) * 32)
#define AP_TMEM_COLS 512
#define AP_SMEM (AG_STAGES * (AG_A_BYTES + AG_B_BYTES) + 2 * AG_BN * 8 * 4 + 256 + 1024)

DEV void ap_epi_bar() { asm volatile("bar.sync 1, %0;" ::"r"(AP_EPI_WARPS * 32) : "memory"); }

__global__ void __launch_bounds__(AP_THREADS, 1)
    k_assoc_gemm_p(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, AssocArgs g) {
  extern __shared__ unsigned char ag_raw[];
  unsigned char* base = (unsigned char*)(((uintptr_t)ag_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* sA = base;
  unsigned char* sB = base + AG_STAGES * AG_A_BYTES;
  float* mbox = (float*)(sB + AG_STAGES * AG_B_BYTES);   // [2][AG_BN][8]
  uint64_t* full = (uint64_t*)(mbox + 2 * AG_BN * 8);
  uint64_t* empty = full + AG_STAGES;
  uint64_t* tfull = empty + AG_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = (uint32_t*)(done + 1);
  __shared__ int sh_fail;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nk = g.dim / AG_BK;
  const int n_mt = (g.n_det + AG_BM - 1) / AG_BM, n_nt = (g.n_mem + AG_BN - 1) / AG_BN;
  const int n_tiles = n_mt * n_nt;
  if (tid == 0) {
    for (int s = 0; s < AG_STAGES; ++s) {
      ag_mbar_init(&full[s], 1);
      ag_mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      ag_mbar_init(&tfull[a], 1);
      ag_mbar_init(&tempty[a], AP_EPI_WARPS);
    }
    ag_mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    sh_fail = 0;
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(ag_smem(tmem_slot)),
                 "r"(AP_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  ag_fence_before();
  __syncthreads();
  ag_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  if (warp == 0) {
    if (lane == 0) {   // TMA producer
      uint32_t it = 0;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
        const int mt = t % n_mt, nt = t / n_mt;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = (int)(it % AG_STAGES);
          const uint32_t ph = (it / AG_STAGES) & 1u;
          if (it >= AG_STAGES && !ag_wait(&empty[s], ph ^ 1u)) { ok = false; break; }
          ag_expect_tx(&full[s], AG_A_BYTES + AG_B_BYTES);
          ag_tma_2d(&tmA, &full[s], sA + s * AG_A_BYTES, kb * AG_BK, mt * AG_BM);
          ag_tma_2d(&tmB, &full[s], sB + s * AG_B_BYTES, kb * AG_BK, nt * AG_BN);
        }
      }
      // drain: the last loads issued must have landed before the CTA exits
      const uint32_t first = it > AG_STAGES ? it - AG_STAGES : 0;
      for (uint32_t j = first; j < it; ++j) ok = ag_wait(&full[j % AG_STAGES], (j / AG_STAGES) & 1u) && ok;
      if (!ok) sh_fail = 1;
    }
  } else if (warp == 1) {
    if (lane == 0) {   // MMA issuer
      uint32_t it = 0, j = 0;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++j) {
        const uint32_t acc = j & 1u;
        if (j >= 2 && !ag_wait(&tempty[acc], ((j >> 1) & 1u) ^ 1u)) { ok = false; break; }
        ag_fence_after();
        const uint32_t dt = tmem + acc * AG_BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = (int)(it % AG_STAGES);
          const uint32_t ph = (it / AG_STAGES) & 1u;
          if (!ag_wait(&full[s], ph)) { ok = false; break; }
          ag_fence_after();
          const uint64_t da = ag_desc(sA + s * AG_A_BYTES), db = ag_desc(sB + s * AG_B_BYTES);
#pragma unroll
          for (int k = 0; k < AG_BK / 16; ++k) ag_mma(dt, da + 2 * k, db + 2 * k, (kb | k) != 0);
          ag_commit(&empty[s]);
        }
        ag_commit(&tfull[acc]);   // also after a failed wait: arrives when the issued MMAs are done
      }
      ag_commit(done);
      if (!ok) sh_fail = 1;
    }
  } else if (warp >= 4) {   // epilogue
    const int ew = warp - 4, quarter = ew & 3, half = ew >> 2;
    const int r = quarter * 32 + lane;
    const float tmin = g.iou_min;
    uint32_t j = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++j) {
      const uint32_t acc = j & 1u;
      const int mt = t % n_mt, nt = t / n_mt;
      const int m0 = mt * AG_BM, n0 = nt * AG_BN;
      // memory boxes of the tile into buffer acc (its previous user, tile j - 2, is done: every
      // epilogue warp passed the barrier of tile j - 1 after it)
      float* mb = mbox + acc * AG_BN * 8;
      for (int c = ew * 32 + lane; c < AG_BN; c += AP_EPI_WARPS * 32) {
        const int jm = n0 + c;
        float b[6] = {0, 0, 0, 0, 0, 0};
        if (jm < g.n_mem)
          for (int k = 0; k < 6; ++k) b[k] = g.mem_box[(size_t)jm * 6 + k];
        float* o = mb + 8 * c;
        for (int k = 0; k < 6; ++k) o[k] = b[k];
        o[6] = ((b[3] - b[0]) * (b[4] - b[1])) * (b[5] - b[2]);
        o[7] = 0.f;
      }
      ap_epi_bar();
      const int d = m0 + r;
      float bx[6] = {0, 0, 0, 0, 0, 0};
      if (d < g.n_det)
        for (int k = 0; k < 6; ++k) bx[k] = g.det_box[(size_t)d * 6 + k];
      const float avol = ((bx[3] - bx[0]) * (bx[4] - bx[1])) * (bx[5] - bx[2]);
      // warp-uniform: tcgen05.ld below is a whole-warp instruction
      const bool got = __all_sync(0xffffffffu, ag_wait(&tfull[acc], (j >> 1) & 1u) ? 1 : 0) != 0;
      ag_fence_after();
      float b1 = -INFINITY, b2 = -INFINITY;
      int i1 = -1;
      const int jlim = g.n_mem - n0;
      const float4* mb4 = (const float4*)mb;
      if (got) {
        for (int c0 = half * (AG_BN / 2); c0 < (half + 1) * (AG_BN / 2); c0 += 16) {
          uint32_t v[16];
          ag_tmem_ld16(tmem + acc * AG_BN + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0, v);
          uint32_t mine = 0;
#pragma unroll
          for (int c = 0; c < 16; ++c) {   // x and y overlap (a superset of the gate)
            const float4 p = mb4[2 * (c0 + c)], q = mb4[2 * (c0 + c) + 1];
            const float e0 = fminf(bx[3], p.w) - fmaxf(bx[0], p.x);
            const float e1 = fminf(bx[4], q.x) - fmaxf(bx[1], p.y);
            mine |= (uint32_t)(e0 > 0.f && e1 > 0.f && c0 + c < jlim) << c;
          }
          const uint32_t any = __reduce_or_sync(0xffffffffu, mine);
          if (!any) continue;
#pragma unroll
          for (int c = 0; c < 16; ++c) {   // the full gate and the top-2, columns in order
            if (!((any >> c) & 1u)) continue;
            const float4 p = mb4[2 * (c0 + c)], q = mb4[2 * (c0 + c) + 1];
            const float e0 = fminf(bx[3], p.w) - fmaxf(bx[0], p.x);
            const float e1 = fminf(bx[4], q.x) - fmaxf(bx[1], p.y);
            const float e2 = fminf(bx[5], q.y) - fmaxf(bx[2], p.z);
            const float inter = (e0 * e1) * e2;
            const float uni = (avol + q.z) - inter;
            const bool pass = ((mine >> c) & 1u) && e2 > 0.f && inter > tmin * uni;
            const float sc = pass ? __uint_as_float(v[c]) : -INFINITY;
            const bool gt = sc > b1;
            b2 = gt ? b1 : fmaxf(b2, sc);
            i1 = gt ? n0 + c0 + c : i1;
            b1 = gt ? sc : b1;
          }
        }
      } else if (lane == 0) {
        sh_fail = 1;
      }
      ag_fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(ag_smem(&tempty[acc])) : "memory");
      if (d < g.n_det) {
        const size_t q = (size_t)d * g.n_tiles + 2 * nt + half;
        g.t_best[q] = i1 >= 0 ? b1 : -INFINITY;
        g.t_second[q] = b2;
        g.t_idx[q] = i1;
      }
    }
  }
  __syncwarp();
  // every issued MMA has completed before TMEM is freed (the issuer's last commit)
  if (!ag_wait(done, 0)) sh_fail = 1;
  ag_fence_before();
  __syncthreads();
  if (tid == 0 && sh_fail) atomicOr(g.err, 1);
  if (warp == 2) {
    ag_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(AP_TMEM_COLS) : "memory");
  }
}
