// Seeded synthetic inputs for the scenemap objprob benchmark configurations.
//
// One header, compiled both by the host compiler (with -ffp-contract=off) and by nvcc
// (with --fmad=false), so that a frame rendered on the CPU and the same frame rendered
// on the GPU are bit-identical: every value below is built from integer hashing and
// IEEE +, -, *, /, sqrt only (no libm transcendental on a per-pixel path).
//
// Scene (config 0/1/4 generator): an axis-aligned room [0,Rx]x[0,Ry]x[0,Rz] holding
// n_boxes axis-aligned boxes standing on the floor.  A pinhole camera renders fp32
// optical depth plus a uint16 instance-label image.  Each visible box face is its own
// label (1 + 3*box + axis, axis 0/1/2 = x/y/z-facing face), so one box yields up to
// three detection fragments, like a segmenter that splits objects into parts; 0 is the
// background (walls, floor, ceiling) unless the scene's shell_labels flag is set: the six
// room faces then get labels of their own (SY_SHELL_LABEL0 + face, face = -x, +x, -y, +y,
// floor, ceiling), like a segmenter that also returns wall, floor and ceiling segments.
// Depth noise is sigma = k*z^2 times a unit-variance Irwin-Hall(12) draw (sum of 12 uniforms
// minus 6), which is reproducible bit for bit.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define SY_HD __host__ __device__ inline
#else
#define SY_HD inline
#endif

#define SY_MAX_BOXES 64
#define SY_SHELL_LABEL0 (1 + 3 * SY_MAX_BOXES)   // first room-face label
#define SY_NLAB (SY_SHELL_LABEL0 + 6)             // label values 0 .. SY_NLAB-1

typedef struct {
  double lo[3], hi[3];
} sy_box;

typedef struct {
  uint64_t seed;
  double room[3];
  int n_boxes;
  sy_box box[SY_MAX_BOXES];
  float noise_k;   // depth noise sigma = noise_k * z^2
  int32_t shell_labels;   // 1: room faces carry labels SY_SHELL_LABEL0 + face (else 0)
} sy_scene;

// The object a label belongs to: box b for its three face labels, SY_MAX_BOXES + face for the
// room faces.  Embeddings (per-object base vector) and classes are keyed by it.
SY_HD int sy_obj_of_label(int label) {
  return label < SY_SHELL_LABEL0 ? (label - 1) / 3 : SY_MAX_BOXES + (label - SY_SHELL_LABEL0);
}

typedef struct {
  int w, h;
  float fx, fy, cx, cy;
} sy_camera;

SY_HD uint64_t sy_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

SY_HD uint64_t sy_hash(uint64_t seed, uint64_t a, uint64_t b, uint64_t c) {
  uint64_t h = sy_mix(c + 0x632BE59BD9B4E019ull);
  h = sy_mix(b * 0xD1B54A32D192ED03ull + h);
  h = sy_mix(a * 0x9E3779B97F4A7C15ull + h);
  return sy_mix(seed ^ h);
}

// uniform in [0, 1) with 53 random bits
SY_HD double sy_u01(uint64_t h) { return (double)(h >> 11) * (1.0 / 9007199254740992.0); }

// unit-variance approximately normal draw: Irwin-Hall sum of 12 uniforms minus 6
SY_HD double sy_gauss(uint64_t seed, uint64_t a, uint64_t b, uint64_t c) {
  double s = 0.0;
  for (uint64_t k = 0; k < 12; ++k) s += sy_u01(sy_hash(seed, a, b, c * 16u + k));
  return s - 6.0;
}

// Ray (origin o, direction d, not normalised) against the scene: returns the ray parameter of
// the first hit (> 1e-9) and its label (room shell: 0, or SY_SHELL_LABEL0 + face with
// shell_labels; 1 + 3*box + axis for box faces).
SY_HD double sy_cast(const sy_scene* S, const double o[3], const double d[3], int* label) {
  // room shell: the exit point of the interior
  double t_best = 1e300;
  int face = 0;
  for (int k = 0; k < 3; ++k) {
    if (d[k] > 0.0) {
      const double t = (S->room[k] - o[k]) / d[k];
      if (t < t_best) { t_best = t; face = 2 * k + 1; }
    } else if (d[k] < 0.0) {
      const double t = (0.0 - o[k]) / d[k];
      if (t < t_best) { t_best = t; face = 2 * k; }
    }
  }
  int lab = S->shell_labels ? SY_SHELL_LABEL0 + face : 0;
  for (int b = 0; b < S->n_boxes; ++b) {
    const sy_box* B = &S->box[b];
    double t0 = -1e300, t1 = 1e300;
    int ax = 0;
    int ok = 1;
    for (int k = 0; k < 3 && ok; ++k) {
      if (d[k] == 0.0) {
        if (o[k] < B->lo[k] || o[k] > B->hi[k]) ok = 0;
        continue;
      }
      double ta = (B->lo[k] - o[k]) / d[k], tb = (B->hi[k] - o[k]) / d[k];
      if (ta > tb) { const double x = ta; ta = tb; tb = x; }
      if (ta > t0) { t0 = ta; ax = k; }
      if (tb < t1) t1 = tb;
    }
    if (!ok || t0 > t1 || t0 <= 1e-9) continue;
    if (t0 < t_best) { t_best = t0; lab = 1 + 3 * b + ax; }
  }
  *label = lab;
  return t_best;
}

// One pixel: optical depth (metres, with noise) and label.  T_mc is map <- camera optical
// (row-major 3x4).  frame_key salts the noise per frame.
SY_HD void sy_pixel(const sy_scene* S, const sy_camera* C, const double T_mc[12], uint64_t frame_key, int u, int v,
                    float* depth, uint16_t* label) {
  const double xn = ((double)u - (double)C->cx) / (double)C->fx;
  const double yn = ((double)v - (double)C->cy) / (double)C->fy;
  const double o[3] = {T_mc[3], T_mc[7], T_mc[11]};
  const double d[3] = {T_mc[0] * xn + T_mc[1] * yn + T_mc[2], T_mc[4] * xn + T_mc[5] * yn + T_mc[6],
                       T_mc[8] * xn + T_mc[9] * yn + T_mc[10]};
  int lab = 0;
  const double t = sy_cast(S, o, d, &lab);   // optical z of the hit = t (camera-frame z of d is 1)
  const double n = sy_gauss(S->seed, frame_key, (uint64_t)v, (uint64_t)u);
  const double z = t + (double)S->noise_k * t * t * n;
  *depth = (float)z;
  *label = (uint16_t)lab;
}

// Embedding element i of a detection of box b in frame f, detection slot k, before
// normalisation: per-box base N(0,1) plus per-detection N(0, sigma).
SY_HD double sy_emb_raw(uint64_t seed, int box, uint64_t frame_key, int k, int i, double sigma) {
  const double base = sy_gauss(seed, 0xE0, (uint64_t)box, (uint64_t)i);
  const double nz = sy_gauss(seed, 0xE1, frame_key * 64u + (uint64_t)k, (uint64_t)i);
  return base + sigma * nz;
}

// float -> bf16 -> float, round to nearest even (NaN not produced by the generator)
SY_HD float sy_bf16_round(float x) {
  union { float f; uint32_t u; } c;
  c.f = x;
  const uint32_t lsb = (c.u >> 16) & 1u;
  c.u = (c.u + 0x7fffu + lsb) & 0xffff0000u;
  return c.f;
}
