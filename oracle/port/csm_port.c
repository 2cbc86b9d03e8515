/* CPU restatement of the correlative scan matcher of BASELINE config 3.
 *
 * TEST INFRASTRUCTURE ONLY (see objprob_port.c): the GPU matcher is checked against this.
 *
 * The reference runs Cartographer's real-time correlative scan matcher (Olson, "Real-Time
 * Correlative Scan Matching", ICRA 2009), configured in src/scene_graph/slam_carto/config/
 * carto_2d.lua:17-21.  Cartographer itself is not vendored in the reference (its README pins
 * rev 877157a, slam_carto/README.md:6), so this is a restatement of the published method, and
 * its parity is unpinned: no reference test fixes matcher outputs.
 *
 * Method, as restated here: the hit points are rotated about the initial pose by each of
 * 2A+1 angles th0 + (j - A) * step and discretised to grid cells once per rotation
 * (cell = floor(world / res), world computed in double as OccGrid::insert does,
 * grid.cpp:207-208); a candidate adds whole-cell offsets (kx, ky) in [-W, W]^2.  Its score is
 * sum_i q(cell_i + (kx, ky)) / (n * 65535) * exp(-(hypot(kx res, ky res) w_t + |(j - A) step| w_r)^2),
 * where q is OccGrid::prob (grid.cpp:261-266: pmin when unseen or outside) quantised to
 * round(p * 65535), so the sum is an exact integer.  Candidates are ordered by rotation, then
 * x offset, then y offset; the first maximum wins.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

static uint16_t q_at(const uint16_t* Q, int W, int H, int X0, int Y0, uint16_t q_out, int ix, int iy) {
  if (ix < X0 || iy < Y0 || ix >= X0 + W || iy >= Y0 + H) return q_out;
  return Q[(size_t)(iy - Y0) * W + (ix - X0)];
}

int op_csm(const uint16_t* Q, int W, int H, int X0, int Y0, uint16_t q_out, float res, const float* hx, const float* hy, int n,
           const double* pose0, int lin_half, int ang_half, double ang_step, double w_t, double w_r, int32_t* best_index,
           double* best_score, double* best_pose) {
  const int nl = 2 * lin_half + 1, nr = 2 * ang_half + 1;
  const double rd = (double)res;
  int* ix = (int*)malloc(sizeof(int) * (size_t)(n > 0 ? n : 1));
  int* iy = (int*)malloc(sizeof(int) * (size_t)(n > 0 ? n : 1));
  double best = -1.0;
  int bi = -1;
  for (int j = 0; j < nr && n > 0; ++j) {
    const double th = pose0[2] + (double)(j - ang_half) * ang_step;
    const double c = cos(th), s = sin(th);
    for (int i = 0; i < n; ++i) {
      const double wx = pose0[0] + c * (double)hx[i] - s * (double)hy[i];
      const double wy = pose0[1] + s * (double)hx[i] + c * (double)hy[i];
      ix[i] = (int)floor(wx / rd);
      iy[i] = (int)floor(wy / rd);
    }
    for (int kx = -lin_half; kx <= lin_half; ++kx)
      for (int ky = -lin_half; ky <= lin_half; ++ky) {
        uint32_t sum = 0;
        for (int i = 0; i < n; ++i) sum += q_at(Q, W, H, X0, Y0, q_out, ix[i] + kx, iy[i] + ky);
        const double t = hypot((double)kx * rd, (double)ky * rd);
        const double a = fabs((double)(j - ang_half) * ang_step);
        const double e = t * w_t + a * w_r;
        const double v = ((double)sum / ((double)n * 65535.0)) * exp(-(e * e));
        if (v > best) {
          best = v;
          bi = (j * nl + (kx + lin_half)) * nl + (ky + lin_half);
        }
      }
  }
  if (n <= 0) {
    bi = (ang_half * nl + lin_half) * nl + lin_half;
    best = 0.0;
  }
  const int j = bi / (nl * nl), r = bi - j * nl * nl, kx = r / nl - lin_half, ky = r % nl - lin_half;
  best_pose[0] = pose0[0] + (double)kx * rd;
  best_pose[1] = pose0[1] + (double)ky * rd;
  best_pose[2] = pose0[2] + (double)(j - ang_half) * ang_step;
  *best_index = bi;
  *best_score = best;
  free(ix);
  free(iy);
  return 0;
}
