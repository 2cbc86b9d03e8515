// Association of observations with memory objects (scenemap src/objmap.cpp:767-810) and the
// pair primitives shared with the merge pass: apCosMax (objprob.cpp:266-285), apContact
// (objprob.cpp:489-504), pairFeatures (objmap.cpp:86-96).
//
// One CTA per (observation, map).  Warps take objects in list order; the box-gap gate is
// evaluated first, and only gate-passing pairs pay for the D-length cosines (double
// accumulation of the fp32 r-vector and the fp16 views against the fp32 detection embedding)
// and the 27-neighbour contact probes of <= 2*contact_samples points.  The per-object P values
// are reduced in list order (first maximum wins, P > same_p), like the reference loop.
#pragma once
#include "dev_util.cuh"

#define ASSOC_THREADS 256
#define SP_MAX 1024
#define ASSOC_GATED 1024

DEV const ObjRec& obj_at(const Batch& B, int m, int pos) { return B.objs[(size_t)m * B.O + B.order[(size_t)m * B.O + pos]]; }
DEV int slot_at(const Batch& B, int m, int pos) { return B.order[(size_t)m * B.O + pos]; }
DEV size_t oglob(const Batch& B, int m, int slot) { return (size_t)m * B.O + slot; }

// contact-cell set membership (ApContactIdx keys, generation-tagged open addressing)
DEV bool contact_has(const Batch& B, size_t cs, uint32_t gen, uint64_t key) {
  const uint64_t* K = B.ckey + cs * B.HCC;
  const uint32_t* G = B.cgen + cs * B.HCC;
  uint32_t h = hmix(key) & (uint32_t)(B.HCC - 1);
  for (int probe = 0; probe < B.HCC; ++probe) {
    if (G[h] != gen) return false;
    if (K[h] == key) return true;
    h = (h + 1) & (uint32_t)(B.HCC - 1);
  }
  return false;
}

// apContact: number of the n sample points (float xyz) whose 27-neighbourhood of `cell` cells
// touches the cloud's contact set.  Warp-level; returns the hit count on every lane.
DEV int contact_hits_warp(const Batch& B, size_t cs, const float* sp, int n, double cell) {
  const CloudRec& C = B.clouds[cs];
  if (n <= 0 || C.cn <= 0) return 0;
  const double inv = 1.0 / cell;
  const int lane = threadIdx.x & 31;
  int hit = 0;
  for (int i = lane; i < n; i += 32) {
    const long long a = (long long)floor((double)sp[3 * i] * inv), b = (long long)floor((double)sp[3 * i + 1] * inv),
                    c = (long long)floor((double)sp[3 * i + 2] * inv);
    if (a < C.clo[0] - 1 || a > C.chi[0] + 1 || b < C.clo[1] - 1 || b > C.chi[1] + 1 || c < C.clo[2] - 1 || c > C.chi[2] + 1) continue;
    if (C.cb_ok) {   // dilated bitset: the cell itself carries the 27-neighbourhood
      const uint32_t* D = B.cbits + cs * 2 * CB_WORDS + CB_WORDS;
      const int x = (int)(a - (C.clo[0] - 1)), y = (int)(b - (C.clo[1] - 1)), z = (int)(c - (C.clo[2] - 1));
      const size_t w = ((size_t)z * C.cb_dy + y) * C.cb_wpr + (x >> 5);
      if (!INB(w, CB_WORDS, 210)) continue;
      hit += (D[w] >> (x & 31)) & 1u;
      continue;
    }
    bool h = false;
    for (int dx = -1; dx <= 1 && !h; ++dx)
      for (int dy = -1; dy <= 1 && !h; ++dy)
        for (int dz = -1; dz <= 1 && !h; ++dz) h = contact_has(B, cs, C.cgen, cell_key3(a + dx, b + dy, c + dz));
    hit += h;
  }
  return warp_sum_i(hit);
}

// apContact with the sample taken on the fly: every stp-th point of cloud `css` (map frame,
// float(org + p), objmap.cpp:1107-1114) against the contact cells of cloud `cst`.  Warp-level.
DEV int contact_hits_cloud_warp(const Batch& B, size_t cst, size_t css, int stp, int n, double cell) {
  const CloudRec& C = B.clouds[cst];
  const CloudRec& S = B.clouds[css];
  if (n <= 0 || C.cn <= 0) return 0;
  const double inv = 1.0 / cell;
  const float4* pts = B.cpts + css * B.cap;
  const uint32_t* Dbits = B.cbits + cst * 2 * CB_WORDS + CB_WORDS;
  int hit = 0;
  for (int q = threadIdx.x & 31; q < n; q += 32) {
    const float4 p = pts[(size_t)q * stp];
    const float x = (float)(S.org[0] + (double)p.x), y = (float)(S.org[1] + (double)p.y), z = (float)(S.org[2] + (double)p.z);
    const long long a = (long long)floor((double)x * inv), b = (long long)floor((double)y * inv), c = (long long)floor((double)z * inv);
    if (a < C.clo[0] - 1 || a > C.chi[0] + 1 || b < C.clo[1] - 1 || b > C.chi[1] + 1 || c < C.clo[2] - 1 || c > C.chi[2] + 1) continue;
    if (C.cb_ok) {
      const int xi = (int)(a - (C.clo[0] - 1)), yi = (int)(b - (C.clo[1] - 1)), zi = (int)(c - (C.clo[2] - 1));
      const size_t w = ((size_t)zi * C.cb_dy + yi) * C.cb_wpr + (xi >> 5);
      if (!INB(w, CB_WORDS, 211)) continue;
      hit += (Dbits[w] >> (xi & 31)) & 1u;
      continue;
    }
    bool h = false;
    for (int dx = -1; dx <= 1 && !h; ++dx)
      for (int dy = -1; dy <= 1 && !h; ++dy)
        for (int dz = -1; dz <= 1 && !h; ++dz) h = contact_has(B, cst, C.cgen, cell_key3(a + dx, b + dy, c + dz));
    hit += h;
  }
  return warp_sum_i(hit);
}

DEV const float* rfrag_of(const Batch& B, size_t og) { return B.rfrag + og * B.D; }
DEV const uint16_t* view_of(const Batch& B, size_t og, int phys) { return B.views + (og * (B.topk + 1) + phys) * B.D; }

// apCosMax of object o against the fp32 vector z (shared or global), warp-level: the fragment
// mean direction r_frag/|r_frag| and each stored fp16 view; returns the max on every lane.
// Every product float*float (or fp16*float) is exact in double; the sums are warp trees.
// When D is a multiple of 128 each lane streams float4 / 4 x fp16 chunks (more loads in flight).
DEV double dot_f32_warp(const float* a, const float* z, int D) {
  const int lane = threadIdx.x & 31;
  double dot = 0;
  if ((D & 127) == 0 && ((((uintptr_t)a) | ((uintptr_t)z)) & 15) == 0) {
    const float4* a4 = (const float4*)a;
    const float4* z4 = (const float4*)z;
#pragma unroll 3
    for (int i = lane; i < D / 4; i += 32) {
      const float4 x = a4[i], y = z4[i];
      dot += (double)x.x * (double)y.x + (double)x.y * (double)y.y + (double)x.z * (double)y.z + (double)x.w * (double)y.w;
    }
  } else {
    for (int i = lane; i < D; i += 32) dot += (double)a[i] * (double)z[i];
  }
  return warp_sum_d(dot);
}
DEV double dot_f16_warp(const uint16_t* q, const float* z, int D) {
  const int lane = threadIdx.x & 31;
  double dot = 0;
  if ((D & 127) == 0 && ((((uintptr_t)q) & 7) | (((uintptr_t)z) & 15)) == 0) {
    const uint2* q4 = (const uint2*)q;
    const float4* z4 = (const float4*)z;
#pragma unroll 3
    for (int i = lane; i < D / 4; i += 32) {
      const uint2 h = q4[i];
      const float4 y = z4[i];
      dot += (double)ref_h2f((uint16_t)(h.x & 0xffffu)) * (double)y.x + (double)ref_h2f((uint16_t)(h.x >> 16)) * (double)y.y +
             (double)ref_h2f((uint16_t)(h.y & 0xffffu)) * (double)y.z + (double)ref_h2f((uint16_t)(h.y >> 16)) * (double)y.w;
    }
  } else {
    for (int i = lane; i < D; i += 32) dot += (double)ref_h2f(q[i]) * (double)z[i];
  }
  return warp_sum_d(dot);
}
DEV double cos_max_warp(const Batch& B, size_t og, const ObjRec& o, const float* z) {
  const int D = B.D;
  double best = -1;
  if (o.nrm_frag > 0) best = smax(best, dot_f32_warp(rfrag_of(B, og), z, D) / sqrt(o.nrm_frag));
  if (o.has_whole && o.nrm_whole > 0) best = smax(best, dot_f32_warp(B.rwhole + og * B.D, z, D) / sqrt(o.nrm_whole));
  for (int v = 0; v < o.n_views; ++v) best = smax(best, dot_f16_warp(view_of(B, og, o.view_slot[v]), z, D));
  return best;
}

// pairFeatures -> P (objmap.cpp:86-96): f0 = contact fraction, f1..f5 = pair_geo, logit, sigmoid
DEV double pair_p(const double alo[3], const double ahi[3], const double apos[3], double contact, const double blo[3],
                  const double bhi[3], const double bpos[3], double cs, const smg_params& P, bool merge, double* f0_out,
                  double f6 = 0.0) {
  double f[7] = {0, 0, 0, 0, 0, 0, 0};
  f[0] = contact;
  pair_geo(alo, ahi, apos, blo, bhi, bpos, cs, P.cos0, f);
  f[6] = f6;   // the merge pair's name-distribution overlap (objmap.cpp:1129-1133), else 0
  if (f0_out) *f0_out = f[0];
  return sigmoid(same_logit(merge ? P.wm : P.w, f));
}

__global__ void __launch_bounds__(ASSOC_THREADS) k_assoc(Batch B) {
  extern __shared__ unsigned char smem_raw[];
  float* zs = (float*)smem_raw;                   // D
  float* sp = zs + B.D;                           // 3 * SP_MAX
  double* pp = (double*)(smem_raw + (((size_t)B.D * 4 + SP_MAX * 12 + 7) & ~(size_t)7));   // O
  __shared__ BlockScratch bs;
  const int a = blockIdx.x, m = B.map0 + blockIdx.y, tid = threadIdx.x;
  const FrameDev& F = B.frames[m];
  const MapRec& R = B.maps[m];
  if (!F.active || a >= R.n_obs) return;
  const smg_params& P = B.p;
  const int det = B.obs_list[(size_t)m * B.max_det + a];
  if (!INB(det, B.max_det, 203)) return;
  ObsRec* O = &B.obs[(size_t)m * B.max_det + det];
  const bool has_z = F.emb != nullptr;
  for (int i = tid; i < B.D; i += blockDim.x) zs[i] = has_z ? emb_at(F.emb, F.emb_dtype, B.D, det, i) : 0.f;
  // contact sample of the observation's cloud candidates (objmap.cpp:776-779)
  const int nc = O->nc;
  const int stp = max(1, nc / max(8, P.contact_samples));
  const int nsp = nc > 0 ? (nc + stp - 1) / stp : 0;
  if (nsp > SP_MAX) {
    if (tid == 0) set_err(&B.maps[m], SMG_E_ARGS);
    return;
  }
  const float* CX = B.cxyz + ((size_t)m * B.max_det + det) * 3 * B.pmax;
  for (int i = tid; i < nsp; i += blockDim.x) {
    sp[3 * i] = CX[3 * (size_t)i * stp];
    sp[3 * i + 1] = CX[3 * (size_t)i * stp + 1];
    sp[3 * i + 2] = CX[3 * (size_t)i * stp + 2];
  }
  __syncthreads();
  const int nobj = R.n_obj;
  const int lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
  // frame-grouping dot products dot(z_b, z_a) with the later observations b (objmap.cpp:992)
  if (has_z)
    for (int b2 = a + 1 + wid; b2 < R.n_obs; b2 += nw) {
      const int det2 = B.obs_list[(size_t)m * B.max_det + b2];
      double dot = 0;
      for (int i = lane; i < B.D; i += 32) dot += (double)emb_at(F.emb, F.emb_dtype, B.D, det2, i) * (double)zs[i];
      dot = warp_sum_d(dot);
      if (lane == 0) B.gdot[((size_t)m * B.max_det + a) * B.max_det + b2] = dot;
    }
  const double gate2 = P.gate * P.gate;
  // box-gap gate of every object, one thread per object; the gated ones go to a list that the
  // warps then work through (the top-1 below reads pp in list order, so the list order is free)
  __shared__ int gl[ASSOC_GATED];   // list position, bit 30: blocked pair (features only)
  __shared__ int ngl, sh_blocked;
  if (tid == 0) { ngl = 0; sh_blocked = 0; }
  __syncthreads();
  // text-model guards (objmap.cpp:792-799): this observation's structure probabilities
  const double o_ps = O->ps, o_pso = O->pso, o_top_p = O->top_p;
  const int o_top = O->top_lab, o_look = O->struct_look;
  {
    double olo[3], ohi[3];
    for (int k = 0; k < 3; ++k) { olo[k] = O->lo[k]; ohi[k] = O->hi[k]; }
    for (int b = tid; b < nobj; b += blockDim.x) {
      if (!INB(b, B.O, 201)) continue;
      const ObjRec& ob = B.objs[oglob(B, m, slot_at(B, m, b))];
      double g2 = 0;
      for (int k = 0; k < 3; ++k) {
        const double g = smax3(0.0, olo[k] - ob.hi[k], ob.lo[k] - ohi[k]);
        g2 += g * g;
      }
      pp[b] = -1.0;
      if (g2 > gate2 || ob.held_by >= 0) continue;   // held objects take no observation (objmap.cpp:785)
      // structure guard: a structure-named object does not take a fragment that is not
      if (o_ps >= 0 && ob.has_post && ob.gp_so >= P.guard_obj && o_ps + o_pso <= P.guard_obs) continue;
      // blocked pairs: a wall-looking fragment and a non-structure object; a flat wall-mounted
      // name grown past its size
      const bool blk = (P.struct_look_block && o_look && ob.has_post && ob.gp_so < 0.5) ||
                       (flat_named(B, ob) && smax(smax(ohi[0], ob.hi[0]) - smin(olo[0], ob.lo[0]),
                                                  smax(ohi[1], ob.hi[1]) - smin(olo[1], ob.lo[1])) > P.flat_max_w);
      if (P.name_veto > 0 && o_top >= 0 && o_top_p >= P.name_veto && ob.top_lab >= 0 && (double)ob.top_p >= P.name_veto &&
          !label_related(B, o_top, ob.top_lab))
        continue;   // names in conflict
      const int q = atomicAdd(&ngl, 1);
      if (q < ASSOC_GATED) gl[q] = b | (blk ? 1 << 30 : 0);
      else set_err(&B.maps[m], SMG_E_ARGS);
    }
  }
  __syncthreads();
  const int ng = ngl < ASSOC_GATED ? ngl : ASSOC_GATED;
  for (int gi = wid; gi < ng; gi += nw) {
    const int b = gl[gi] & ~(1 << 30);
    const bool blk = (gl[gi] >> 30) & 1;
    const int slot = slot_at(B, m, b);
    const size_t og = oglob(B, m, slot);
    const ObjRec& ob = B.objs[og];
    if (!INB(slot, B.O, 202)) continue;
    const double cs = has_z ? cos_max_warp(B, og, ob, zs) : -2.0;
    if (has_z && lane == 0) wk_add(&B.maps[m], SMG_WK_VEC16, (ob.nrm_frag > 0 ? 2 : 0) + ob.n_views);
    const size_t cslot = cglob(B, m, ob.cloud_slot);
    const int hits = contact_hits_warp(B, cslot, sp, nsp, P.contact_cell);
    if (lane == 0) {
      const double contact = (nsp > 0 && B.clouds[cslot].cn > 0) ? (double)hits / (double)nsp : 0.0;
      double f0;
      const double p = pair_p(O->lo, O->hi, O->pos, contact, ob.lo, ob.hi, ob.pos, cs, P, false, &f0);
      if (f0 >= 0.3 || p >= 0.2) B.touched[(size_t)m * B.O + b] = 1;
      if (blk) {   // features (touched) only; a pair that would have matched blocks the fragment
        if (p >= P.same_p) sh_blocked = 1;
      } else {
        pp[b] = p;
      }
    }
  }
  __syncthreads();
  // first maximum in list order with P > same_p; count P >= same_p (objmap.cpp:780-806)
  double bp = -2.0;
  int bi = -1, ns = 0;
  for (int b = tid; b < nobj; b += blockDim.x) {
    const double p = pp[b];
    ns += p >= P.same_p;
    if (p > bp) { bp = p; bi = b; }
  }
  // combine (max p, then smallest index)
  for (int o = 16; o > 0; o >>= 1) {
    const double p2 = __shfl_xor_sync(0xffffffffu, bp, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    if (p2 > bp || (p2 == bp && i2 >= 0 && (bi < 0 || i2 < bi))) { bp = p2; bi = i2; }
  }
  __shared__ double wbp[32];
  __shared__ int wbi[32];
  if (lane == 0) { wbp[wid] = bp; wbi[wid] = bi; }
  const int nsame = block_sum_i(ns, bs);
  if (tid == 0) {
    double best = P.same_p;
    int to = -1;
    double mp = -2.0;
    int mi = -1;
    for (int w = 0; w < nw; ++w)
      if (wbp[w] > mp || (wbp[w] == mp && wbi[w] >= 0 && (mi < 0 || wbi[w] < mi))) { mp = wbp[w]; mi = wbi[w]; }
    if (mi >= 0 && mp > best) to = mi;
    O->obs_to = to;
    O->n_same = nsame;
    O->blocked = sh_blocked;
  }
}
