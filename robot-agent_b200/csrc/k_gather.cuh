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
// One CTA per (image row, map): the row's pixel masks are built from the boxes in shared memory,
// then the masked pixels are copied in 16-byte chunks.
#pragma once
#include "dev_util.cuh"

#define GATHER_THREADS 256
#define GATHER_WMAX 2048   // widest frame the row masks cover

__global__ void __launch_bounds__(GATHER_THREADS) k_gather(Batch B) {
  __shared__ uint32_t dmask[GATHER_WMAX / 32], lmask[GATHER_WMAX / 32];
  const int v = blockIdx.x, m = B.map0 + blockIdx.y, tid = threadIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active || !F.depth_host || v >= F.h) return;
  const int W = F.w, nw = (W + 31) >> 5;
  if (W > GATHER_WMAX) return;   // rejected on the host
  // whole rows (copied by the copy engines): makeScan's and markView's sample rows
  const int step = max(1, (int)llround(F.w / 160.0));
  const int stp = max(1, F.w / 32);
  const bool full = v % step == 0 || (v >= stp / 2 && (v - stp / 2) % stp == 0);
  for (int i = tid; i < nw; i += blockDim.x) { dmask[i] = 0u; lmask[i] = 0u; }   // whole rows come by copy
  __syncthreads();
  // detection boxes: depth over [u0, u1] on rows [v0, v1], labels one pixel wider on both axes
  auto set_bits = [](uint32_t* mask, int lo, int hi) {   // bits lo..hi, a word at a time
    for (int u = lo; u <= hi;) {
      const int w = u >> 5, e = min(hi, (w << 5) + 31);
      const uint32_t bits = (e - u == 31) ? 0xffffffffu : (((1u << (e - u + 1)) - 1u) << (u & 31));
      atomicOr(&mask[w], bits);
      u = e + 1;
    }
  };
  for (int k = tid; k < F.n_det; k += blockDim.x) {
    int u0, u1, v0, v1;
    det_scan_box(F, k, &u0, &u1, &v0, &v1);
    if (u1 < u0 || v < v0 - 1 || v > v1 + 1) continue;
    set_bits(lmask, max(0, u0 - 1), min(W - 1, u1 + 1));
    if (!full && v >= v0 && v <= v1) set_bits(dmask, u0, u1);
  }
  __syncthreads();
  const size_t row = (size_t)v * W;
  float* dd = const_cast<float*>(F.depth) + row;
  uint16_t* dl = const_cast<uint16_t*>(F.label) + row;
  const float* sd = F.depth_host + row;
  const uint16_t* sl = F.label_host ? F.label_host + row : nullptr;
  // 16-byte chunks (4 depth or 8 label pixels) whenever the rows allow it: a chunk with any
  // pixel needed is moved whole, so every read across PCIe is a full 16-byte request
  const bool dvec = (W & 3) == 0 && ((((uintptr_t)sd) | ((uintptr_t)dd)) & 15) == 0;
  const bool lvec = sl && (W & 7) == 0 && ((((uintptr_t)sl) | ((uintptr_t)dl)) & 15) == 0;
  const int nd4 = dvec ? W >> 2 : 0, nl8 = lvec ? W >> 3 : 0;
  int moved = 0;   // bytes read from host memory
  for (int c = tid; c < nd4 + nl8; c += blockDim.x) {
    if (c < nd4) {
      if ((dmask[c >> 3] >> ((c & 7) << 2)) & 0xfu) { ((uint4*)dd)[c] = ((const uint4*)sd)[c]; moved += 16; }
    } else {
      const int q = c - nd4;
      if ((lmask[q >> 2] >> ((q & 3) << 3)) & 0xffu) { ((uint4*)dl)[q] = ((const uint4*)sl)[q]; moved += 16; }
    }
  }
  for (int u = tid; u < W; u += blockDim.x) {   // rows that do not allow 16-byte chunks
    const uint32_t bit = 1u << (u & 31);
    if (!dvec && (dmask[u >> 5] & bit)) { dd[u] = sd[u]; moved += 4; }
    if (sl && !lvec && (lmask[u >> 5] & bit)) { dl[u] = sl[u]; moved += 2; }
  }
  moved = __reduce_add_sync(0xffffffffu, moved);
  if ((tid & 31) == 0 && moved) wk_add(&B.maps[m], SMG_WK_H2D, moved);
}
