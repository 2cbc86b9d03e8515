// Host-input gather: with pinned (device-accessible) host frames, the chain's staging images
// receive only the pixels the chain reads, fetched by the SMs straight from host memory, instead
// of whole-frame copies.  Which pixels a kernel reads is fixed by the frame's descriptor alone:
//  - k_obs: depth over each detection's scan box [u0, u1] x [v0, v1] and, for the label-image
//    form, labels over that box grown by one pixel (the 4-neighbour erosion), with
//    u0 = max(0, int(x0 * sx) - 1) etc. (objmap.cpp:648-652, det_scan_box as k_obs uses it);
//  - k_grid: the depth rows v = j * step (makeScan's grid, scan.cpp:233-251);
//  - k_markview: the depth rows v = stp/2 + j * stp (objmap.cpp:219-245).
// Those whole rows travel by strided copies on the copy engines, beside this kernel; the kernel
// moves the box pixels of the other rows and every label pixel.
// k_absent reads depth at the projections of object clouds, which depend on the map state; it
// reads those few pixels from the host frame directly (FrameDev::depth_host).
// A few CTAs per map, each walking the map's rows GATHER_ROWS at a time: the rows' pixel masks
// are built from the boxes in shared memory, then every thread issues all its 16-byte host reads
// of the GATHER_ROWS rows before storing any, so one PCIe round trip moves a CTA's rows.  Few,
// long-lived CTAs keep the reads going while the previous keyframe's chain holds most SMs.
#pragma once
#include "dev_util.cuh"

#define GATHER_THREADS 256
#define GATHER_WMAX 2048   // widest frame the row masks cover
#ifndef GATHER_ROWS
#define GATHER_ROWS 16     // rows per pass of a CTA
#endif
#ifndef GATHER_CTAS
#define GATHER_CTAS 1      // CTAs per map
#endif
#ifndef GATHER_ILP
#define GATHER_ILP 16      // 16-byte reads in flight per thread
#endif

__global__ void __launch_bounds__(GATHER_THREADS) k_gather(Batch B) {
  __shared__ uint32_t dmask[GATHER_ROWS][GATHER_WMAX / 32], lmask[GATHER_ROWS][GATHER_WMAX / 32];
  const int m = B.map0 + blockIdx.y, tid = threadIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active || !F.depth_host) return;
  const int W = F.w, H = F.h, nw = (W + 31) >> 5;
  if (W > GATHER_WMAX) return;   // rejected on the host
  // whole rows (copied by the copy engines): makeScan's and markView's sample rows
  const int step = max(1, (int)llround(F.w / 160.0));
  const int stp = max(1, F.w / 32);
  auto set_bits = [](uint32_t* mask, int lo, int hi) {   // bits lo..hi, a word at a time
    for (int u = lo; u <= hi;) {
      const int w = u >> 5, e = min(hi, (w << 5) + 31);
      const uint32_t bits = (e - u == 31) ? 0xffffffffu : (((1u << (e - u + 1)) - 1u) << (u & 31));
      atomicOr(&mask[w], bits);
      u = e + 1;
    }
  };
  float* d0 = const_cast<float*>(F.depth);
  uint16_t* l0 = const_cast<uint16_t*>(F.label);
  const float* sd0 = F.depth_host;
  const uint16_t* sl0 = F.label_host;
  // 16-byte chunks (4 depth or 8 label pixels) whenever the rows allow it: a chunk with any
  // pixel needed is moved whole, so every read across PCIe is a full 16-byte request
  const bool dvec = (W & 3) == 0 && ((((uintptr_t)sd0) | ((uintptr_t)d0)) & 15) == 0;
  const bool lvec = sl0 && (W & 7) == 0 && ((((uintptr_t)sl0) | ((uintptr_t)l0)) & 15) == 0;
  const int nd4 = dvec ? W >> 2 : 0, nl8 = lvec ? W >> 3 : 0, per = nd4 + nl8;
  int moved = 0;   // bytes read from host memory
  for (int vb = blockIdx.x * GATHER_ROWS; vb < H; vb += gridDim.x * GATHER_ROWS) {
    for (int i = tid; i < GATHER_ROWS * nw; i += blockDim.x) {
      dmask[i / nw][i % nw] = 0u;
      lmask[i / nw][i % nw] = 0u;
    }
    __syncthreads();
    // detection boxes: depth over [u0, u1] on rows [v0, v1], labels one pixel wider on both axes
    for (int t = tid; t < F.n_det * GATHER_ROWS; t += blockDim.x) {
      const int k = t / GATHER_ROWS, r = t - k * GATHER_ROWS, v = vb + r;
      if (v >= H) continue;
      int u0, u1, v0, v1;
      det_scan_box(F, k, &u0, &u1, &v0, &v1);
      if (u1 < u0 || v < v0 - 1 || v > v1 + 1) continue;
      const bool full = v % step == 0 || (v >= stp / 2 && (v - stp / 2) % stp == 0);
      set_bits(lmask[r], max(0, u0 - 1), min(W - 1, u1 + 1));
      if (!full && v >= v0 && v <= v1) set_bits(dmask[r], u0, u1);
    }
    __syncthreads();
    const int tot = GATHER_ROWS * per;
    for (int c0 = 0; c0 < tot; c0 += GATHER_ILP * blockDim.x) {
      uint4 val[GATHER_ILP];
      uint4* dst[GATHER_ILP];
#pragma unroll
      for (int j = 0; j < GATHER_ILP; ++j) {   // all reads first
        dst[j] = nullptr;
        const int c = c0 + j * blockDim.x + tid;
        if (c >= tot) continue;
        const int r = c / per, q = c - r * per, v = vb + r;
        if (v >= H) continue;
        const size_t row = (size_t)v * W;
        if (q < nd4) {
          if ((dmask[r][q >> 3] >> ((q & 7) << 2)) & 0xfu) {
            dst[j] = (uint4*)(d0 + row) + q;
            val[j] = ((const uint4*)(sd0 + row))[q];
          }
        } else {
          const int q8 = q - nd4;
          if ((lmask[r][q8 >> 2] >> ((q8 & 3) << 3)) & 0xffu) {
            dst[j] = (uint4*)(l0 + row) + q8;
            val[j] = ((const uint4*)(sl0 + row))[q8];
          }
        }
      }
#pragma unroll
      for (int j = 0; j < GATHER_ILP; ++j)
        if (dst[j]) { *dst[j] = val[j]; moved += 16; }
    }
    for (int r = 0; r < GATHER_ROWS && (!dvec || (sl0 && !lvec)); ++r) {   // rows that do not allow 16-byte chunks
      const int v = vb + r;
      if (v >= H) break;
      const size_t row = (size_t)v * W;
      for (int u = tid; u < W; u += blockDim.x) {
        const uint32_t bit = 1u << (u & 31);
        if (!dvec && (dmask[r][u >> 5] & bit)) { d0[row + u] = sd0[row + u]; moved += 4; }
        if (sl0 && !lvec && (lmask[r][u >> 5] & bit)) { l0[row + u] = sl0[row + u]; moved += 2; }
      }
    }
    __syncthreads();   // the masks are rebuilt for the next rows
  }
  moved = __reduce_add_sync(0xffffffffu, moved);
  if ((tid & 31) == 0 && moved) wk_add(&B.maps[m], SMG_WK_H2D, moved);
}
