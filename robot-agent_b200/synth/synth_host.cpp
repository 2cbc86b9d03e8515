// Host side of the synthetic scene generator (see synth.h): box placement, camera
// trajectory, frame rendering, detection extraction from the label image and the
// per-detection embeddings.  Exposed as a plain C API (ctypes) for tests and bench.py.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "synth.h"

extern "C" {

// Place n_boxes non-overlapping axis-aligned boxes on the floor of a room of size rx x ry x rz.
int sy_scene_make(uint64_t seed, int n_boxes, double rx, double ry, double rz, float noise_k, double size_lo, double size_hi,
                  double h_lo, double h_hi, sy_scene* out) {
  if (!out || n_boxes < 0 || n_boxes > SY_MAX_BOXES) return -1;
  memset(out, 0, sizeof(*out));
  out->seed = seed;
  out->room[0] = rx;
  out->room[1] = ry;
  out->room[2] = rz;
  out->noise_k = noise_k;
  uint64_t ctr = 0;
  auto u = [&]() { return sy_u01(sy_hash(seed, 0xB0, ctr++, 0)); };
  int placed = 0;
  for (int tries = 0; placed < n_boxes && tries < 100000; ++tries) {
    const double sx = size_lo + (size_hi - size_lo) * u(), sy = size_lo + (size_hi - size_lo) * u();
    const double sz = h_lo + (h_hi - h_lo) * u();
    const double x0 = 0.3 + (rx - 0.6 - sx) * u(), y0 = 0.3 + (ry - 0.6 - sy) * u();
    bool ok = true;
    for (int b = 0; b < placed && ok; ++b) {
      const sy_box& B = out->box[b];
      const double g = 0.15;
      ok = x0 + sx + g < B.lo[0] || B.hi[0] + g < x0 || y0 + sy + g < B.lo[1] || B.hi[1] + g < y0;
    }
    if (!ok) continue;
    sy_box& B = out->box[placed++];
    B.lo[0] = x0; B.lo[1] = y0; B.lo[2] = 0.0;
    B.hi[0] = x0 + sx; B.hi[1] = y0 + sy; B.hi[2] = sz;
  }
  out->n_boxes = placed;
  return placed;
}

// Base trajectory (x, y, th per frame): seeded random walk at `speed` m/s that keeps `clear`
// metres from walls and box footprints; the camera heading looks towards the room centre
// with a slow sinusoidal sweep.
int sy_traj(const sy_scene* S, int n_frames, double dt, double speed, double clear, double* poses) {
  if (!S || n_frames <= 0 || !poses) return -1;
  auto is_free = [&](double x, double y) {
    if (x < clear || y < clear || x > S->room[0] - clear || y > S->room[1] - clear) return false;
    for (int b = 0; b < S->n_boxes; ++b) {
      const sy_box& B = S->box[b];
      if (x > B.lo[0] - clear && x < B.hi[0] + clear && y > B.lo[1] - clear && y < B.hi[1] + clear) return false;
    }
    return true;
  };
  uint64_t ctr = 0;
  auto u = [&]() { return sy_u01(sy_hash(S->seed, 0xC0, ctr++, 0)); };
  double x = 0, y = 0;
  for (int t = 0; t < 100000; ++t) {
    x = S->room[0] * u();
    y = S->room[1] * u();
    if (is_free(x, y)) break;
  }
  double hd = 2.0 * M_PI * u();
  const double phase = 2.0 * M_PI * u();
  for (int f = 0; f < n_frames; ++f) {
    hd += 0.3 * sy_gauss(S->seed, 0xC1, (uint64_t)f, 0);
    const double step = speed * dt;
    bool moved = false;
    for (int k = 0; k < 24 && !moved; ++k) {
      const double nx = x + step * cos(hd), ny = y + step * sin(hd);
      if (is_free(nx, ny)) {
        x = nx;
        y = ny;
        moved = true;
      } else {
        hd += 0.5 * M_PI + (u() - 0.5);
      }
    }
    const double look = atan2(0.5 * S->room[1] - y, 0.5 * S->room[0] - x) + 0.8 * sin(0.23 * f * dt + phase);
    poses[3 * f] = x;
    poses[3 * f + 1] = y;
    poses[3 * f + 2] = look;
  }
  return 0;
}

// Camera mount: base <- camera optical (row-major 3x4, float like the reference FK output).
// Camera at (fwd, 0, height) in the base frame, optical z forward and pitched down by pitch_deg.
void sy_rig_T_bc(float fwd, float height, float pitch_deg, float T_bc[12]) {
  const double p = pitch_deg * M_PI / 180.0, sp = sin(p), cp = cos(p);
  const double R[12] = {0, -sp, cp, fwd, -1, 0, 0, 0, 0, -cp, -sp, height};
  for (int i = 0; i < 12; ++i) T_bc[i] = (float)R[i];
}

// map <- camera optical from the base pose and the mount, by the same arithmetic as the
// reference's keyframe glue (scenemap capi.cpp:836-843).
void sy_T_mc(const double pose[3], const float B[12], double T_mc[12]) {
  const double cs = cos(pose[2]), sn = sin(pose[2]);
  for (int r = 0; r < 3; ++r) {
    const double R0 = r == 0 ? cs : (r == 1 ? sn : 0), R1 = r == 0 ? -sn : (r == 1 ? cs : 0), R2 = r == 2 ? 1 : 0;
    for (int k = 0; k < 4; ++k) T_mc[r * 4 + k] = R0 * B[k] + R1 * B[4 + k] + R2 * B[8 + k];
  }
  T_mc[3] += pose[0];
  T_mc[7] += pose[1];
}

void sy_render(const sy_scene* S, const sy_camera* C, const double T_mc[12], uint64_t frame_key, float* depth, uint16_t* label) {
  for (int v = 0; v < C->h; ++v)
    for (int u = 0; u < C->w; ++u) sy_pixel(S, C, T_mc, frame_key, u, v, depth + (size_t)v * C->w + u, label + (size_t)v * C->w + u);
}

// Detections from a label image: one per label value with >= min_px pixels, ordered by pixel
// count (descending, ties by label).  box = [umin, vmin, umax + 1, vmax + 1] in pixels.
int sy_dets(const uint16_t* label, int w, int h, int min_px, int max_det, uint16_t* det_label, float* box, int32_t* cls, float* score) {
  const int L = SY_NLAB;
  std::vector<int> cnt(L, 0), u0(L, w), v0(L, h), u1(L, -1), v1(L, -1);
  for (int v = 0; v < h; ++v)
    for (int u = 0; u < w; ++u) {
      const int l = label[(size_t)v * w + u];
      if (l <= 0 || l >= L) continue;
      ++cnt[l];
      u0[l] = std::min(u0[l], u); u1[l] = std::max(u1[l], u);
      v0[l] = std::min(v0[l], v); v1[l] = std::max(v1[l], v);
    }
  std::vector<int> ids;
  for (int l = 1; l < L; ++l) if (cnt[l] >= min_px) ids.push_back(l);
  std::stable_sort(ids.begin(), ids.end(), [&](int a, int b) { return cnt[a] > cnt[b]; });
  const int n = std::min<int>(int(ids.size()), max_det);
  for (int k = 0; k < n; ++k) {
    const int l = ids[size_t(k)];
    det_label[k] = (uint16_t)l;
    box[4 * k] = (float)u0[l];
    box[4 * k + 1] = (float)v0[l];
    box[4 * k + 2] = (float)(u1[l] + 1);
    box[4 * k + 3] = (float)(v1[l] + 1);
    cls[k] = sy_obj_of_label(l) % 16;
    score[k] = 0.5f + 0.5f * std::min(1.f, (float)cnt[l] / 20000.f);
  }
  return n;
}

// L2-normalised embeddings (n x D) for detections with the given labels; bf16 != 0 rounds each
// element to bf16 after normalisation (the value the reference then reads as float).
void sy_embed(const sy_scene* S, uint64_t frame_key, int n, const uint16_t* det_label, int D, double sigma, int bf16, float* out) {
  std::vector<double> v((size_t)D);
  for (int k = 0; k < n; ++k) {
    const int box = sy_obj_of_label(det_label[k]);
    double s = 0;
    for (int i = 0; i < D; ++i) {
      v[(size_t)i] = sy_emb_raw(S->seed, box, frame_key, k, i, sigma);
      s += v[(size_t)i] * v[(size_t)i];
    }
    const double inv = 1.0 / sqrt(s);
    for (int i = 0; i < D; ++i) {
      const float f = (float)(v[(size_t)i] * inv);
      out[(size_t)k * D + i] = bf16 ? sy_bf16_round(f) : f;
    }
  }
}

}  // extern "C"
