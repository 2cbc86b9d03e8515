// Device side of the synthetic generator (synth.h): renders frames, label statistics and
// detection embeddings directly in HBM, for benchmark inputs.  Not on the measured path.
// The per-pixel render is the same function as the host generator, and embeddings are
// normalised with the host's sum order (one thread adds the squares in index order), so the
// device renders bit for bit the frames the host generator renders.
#include <stdint.h>

#include "synth.h"

// frames f of maps m: T_all[(f*M + m)*12], keys[f*M + m]; output image (f*M + m)
__global__ void sy_render_batch_kernel(const sy_scene* __restrict__ scenes, sy_camera Cm, const double* __restrict__ T_all,
                                       const uint64_t* __restrict__ keys, int M, int n_img, float* __restrict__ depth,
                                       uint16_t* __restrict__ label) {
  const int img = blockIdx.y;
  if (img >= n_img) return;
  const sy_scene* S = &scenes[img % M];
  const size_t WH = (size_t)Cm.w * Cm.h;
  double T[12];
  for (int k = 0; k < 12; ++k) T[k] = T_all[12 * (size_t)img + k];
  for (size_t p = blockIdx.x * (size_t)blockDim.x + threadIdx.x; p < WH; p += (size_t)gridDim.x * blockDim.x) {
    const int u = (int)(p % Cm.w), v = (int)(p / Cm.w);
    sy_pixel(S, &Cm, T, keys[img], u, v, depth + img * WH + p, label + img * WH + p);
  }
}

// per image and label: count, umin, vmin, umax, vmax (stats[img][SY_NLAB][5])
__global__ void sy_label_stats_kernel(const uint16_t* __restrict__ label, int w, int h, int n_img, int* __restrict__ stats) {
  __shared__ int s[SY_NLAB * 5];
  const int img = blockIdx.y;
  if (img >= n_img) return;
  for (int i = threadIdx.x; i < SY_NLAB; i += blockDim.x) {
    s[5 * i] = 0; s[5 * i + 1] = w; s[5 * i + 2] = h; s[5 * i + 3] = -1; s[5 * i + 4] = -1;
  }
  __syncthreads();
  const size_t WH = (size_t)w * h;
  const uint16_t* L = label + img * WH;
  for (size_t p = blockIdx.x * (size_t)blockDim.x + threadIdx.x; p < WH; p += (size_t)gridDim.x * blockDim.x) {
    const int l = L[p];
    if (l <= 0 || l >= SY_NLAB) continue;
    const int u = (int)(p % w), v = (int)(p / w);
    atomicAdd(&s[5 * l], 1);
    atomicMin(&s[5 * l + 1], u); atomicMin(&s[5 * l + 2], v);
    atomicMax(&s[5 * l + 3], u); atomicMax(&s[5 * l + 4], v);
  }
  __syncthreads();
  int* o = stats + (size_t)img * SY_NLAB * 5;
  for (int i = threadIdx.x; i < SY_NLAB; i += blockDim.x) {
    atomicAdd(&o[5 * i], s[5 * i]);
    atomicMin(&o[5 * i + 1], s[5 * i + 1]); atomicMin(&o[5 * i + 2], s[5 * i + 2]);
    atomicMax(&o[5 * i + 3], s[5 * i + 3]); atomicMax(&o[5 * i + 4], s[5 * i + 4]);
  }
}

__global__ void sy_stats_init_kernel(int* stats, int n_img, int w, int h) {
  const size_t n = (size_t)n_img * SY_NLAB;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    stats[5 * i] = 0; stats[5 * i + 1] = w; stats[5 * i + 2] = h; stats[5 * i + 3] = -1; stats[5 * i + 4] = -1;
  }
}

// one block per detection: desc[5*j] = map, object (sy_obj_of_label), det slot k, frame key
// (as two ints: lo, hi).  The raw values are staged in shared memory and their squares summed in
// index order by one thread, as the host generator does, so the normalised values are the same
// floats.
#define SY_EMB_DMAX 2048
__global__ void sy_embed_kernel(const sy_scene* __restrict__ scenes, const int* __restrict__ desc, int n, int D, double sigma,
                                int bf16, void* __restrict__ out) {
  const int j = blockIdx.x;
  if (j >= n) return;
  const int m = desc[5 * j], box = desc[5 * j + 1], k = desc[5 * j + 2];
  const uint64_t key = (uint64_t)(uint32_t)desc[5 * j + 3] | ((uint64_t)(uint32_t)desc[5 * j + 4] << 32);
  const uint64_t seed = scenes[m].seed;
  __shared__ double v[SY_EMB_DMAX];
  __shared__ double inv;
  for (int i = threadIdx.x; i < D; i += blockDim.x) v[i] = sy_emb_raw(seed, box, key, k, i, sigma);
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0;
    for (int i = 0; i < D; ++i) s += v[i] * v[i];
    inv = 1.0 / sqrt(s);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float f = (float)(v[i] * inv);
    if (bf16) ((uint16_t*)out)[(size_t)j * D + i] = (uint16_t)(__float_as_uint(sy_bf16_round(f)) >> 16);
    else ((float*)out)[(size_t)j * D + i] = f;
  }
}

// Detector bit masks on an s-pixel grid (synth.py label_masks): cell (i, j) of detection k of
// image img is set when the label at pixel (s i + s/2, s j + s/2) is that detection's label.
// One thread per output word (32 cells, LSB first).
__global__ void sy_masks_kernel(const uint16_t* __restrict__ label, int w, int h, int s, const uint16_t* __restrict__ det_label,
                                const int* __restrict__ n_det, int max_det, uint32_t* __restrict__ out) {
  const int img = blockIdx.z, k = blockIdx.y;
  const int MW = w / s, MH = h / s, words = (MW * MH + 31) / 32;
  const int wd = blockIdx.x * blockDim.x + threadIdx.x;
  if (wd >= words || k >= max_det) return;
  uint32_t v = 0;
  if (k < n_det[img]) {
    const uint16_t L = det_label[(size_t)img * max_det + k];
    const uint16_t* lab = label + (size_t)img * w * h;
    for (int b = 0; b < 32; ++b) {
      const int q = wd * 32 + b;
      if (q >= MW * MH) break;
      const int i = q % MW, j = q / MW;
      if (lab[(size_t)(s * j + s / 2) * w + (s * i + s / 2)] == L) v |= 1u << b;
    }
  }
  out[((size_t)img * max_det + k) * words + wd] = v;
}

extern "C" {

int sy_masks_device(const uint16_t* label_dev, int w, int h, int s, const uint16_t* det_label_dev, const int* n_det_dev, int max_det,
                    int n_img, uint32_t* out_dev, void* stream) {
  if (s <= 0 || w / s <= 0 || h / s <= 0 || max_det <= 0 || n_img <= 0) return -1;
  const int words = ((w / s) * (h / s) + 31) / 32;
  sy_masks_kernel<<<dim3((words + 255) / 256, max_det, n_img), 256, 0, (cudaStream_t)stream>>>(label_dev, w, h, s, det_label_dev, n_det_dev,
                                                                                              max_det, out_dev);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int sy_render_batch_device(const sy_scene* scenes_dev, const sy_camera* C, const double* T_dev, const uint64_t* keys_dev, int M,
                           int n_img, float* depth_dev, uint16_t* label_dev, void* stream) {
  dim3 grid(296, n_img);
  sy_render_batch_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(scenes_dev, *C, T_dev, keys_dev, M, n_img, depth_dev, label_dev);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int sy_label_stats_device(const uint16_t* label_dev, int w, int h, int n_img, int* stats_dev, void* stream) {
  sy_stats_init_kernel<<<256, 256, 0, (cudaStream_t)stream>>>(stats_dev, n_img, w, h);
  sy_label_stats_kernel<<<dim3(16, n_img), 512, 0, (cudaStream_t)stream>>>(label_dev, w, h, n_img, stats_dev);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int sy_embed_device(const sy_scene* scenes_dev, const int* desc_dev, int n, int D, double sigma, int bf16, void* out_dev, void* stream) {
  if (n <= 0) return 0;
  if (D <= 0 || D > SY_EMB_DMAX) return -1;
  sy_embed_kernel<<<n, 256, 0, (cudaStream_t)stream>>>(scenes_dev, desc_dev, n, D, sigma, bf16, out_dev);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int sy_nlab(void) { return SY_NLAB; }

}  // extern "C"
