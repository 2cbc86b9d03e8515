// Device renderer of the synthetic box room (synth.h): the same per-pixel function as the
// host generator, for producing benchmark inputs directly in HBM.  Not on the measured path.
#include <stdint.h>

#include "synth.h"

__global__ void sy_render_kernel(sy_scene S, sy_camera Cm, const double* __restrict__ T_all, const uint64_t* __restrict__ keys,
                                 int n_frames, float* __restrict__ depth, uint16_t* __restrict__ label) {
  const int f = blockIdx.y;
  if (f >= n_frames) return;
  const size_t WH = (size_t)Cm.w * Cm.h;
  double T[12];
  for (int k = 0; k < 12; ++k) T[k] = T_all[12 * f + k];
  for (size_t p = blockIdx.x * (size_t)blockDim.x + threadIdx.x; p < WH; p += (size_t)gridDim.x * blockDim.x) {
    const int u = (int)(p % Cm.w), v = (int)(p / Cm.w);
    sy_pixel(&S, &Cm, T, keys[f], u, v, depth + f * WH + p, label + f * WH + p);
  }
}

extern "C" int sy_render_device(const sy_scene* S, const sy_camera* C, const double* T_dev, const uint64_t* keys_dev, int n_frames,
                                float* depth_dev, uint16_t* label_dev, void* stream) {
  dim3 grid(148, n_frames);
  sy_render_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(*S, *C, T_dev, keys_dev, n_frames, depth_dev, label_dev);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
