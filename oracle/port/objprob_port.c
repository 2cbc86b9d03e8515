/* CPU restatement of the scenemap objprob primitives on the B200 path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity tests, __graft_entry__.smoke() and bench.py's CPU
 * baseline may load this (as oracle/_ref/libport.so) to check the CUDA kernels; the product
 * library never links or calls it.
 *
 * Each function restates one reference routine (file:line within src/scene_graph/scenemap);
 * the arithmetic follows the reference's order and types so results are bit-identical with
 * it when both are compiled without FMA contraction (-ffp-contract=off here, baseline x86-64
 * in the reference build).  Pinned by tests/test_oracle_port.py against the reference's
 * known-answer tests (tests/test_objprob.cpp) and against golden outputs of the reference
 * itself (tests/golden/).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* splitmix64 step (objprob.cpp:116-121) */
static uint64_t sm_next(uint64_t* s) {
  uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* apSeed (objprob.cpp:125-128): mix two words, one splitmix step */
uint64_t op_ap_seed(uint64_t a, uint64_t b) {
  uint64_t s = a * 0x9E3779B97F4A7C15ull ^ (b + 0x632BE59BD9B4E019ull);
  return sm_next(&s);
}

/* f2h (objprob.cpp:12-29): the reference's own fp32 -> fp16 rounding (round half up on the
 * dropped 13 bits; subnormals rounded, tiny values flushed to signed zero, overflow -> inf) */
uint16_t op_f2h(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sgn = (x >> 16) & 0x8000u;
  int32_t ex = (int32_t)((x >> 23) & 0xffu) - 112; /* rebias 127 -> 15 */
  uint32_t man = x & 0x7fffffu;
  if (ex <= 0) {
    if (ex < -10) return (uint16_t)sgn;
    man |= 0x800000u;
    const int shift = 14 - ex;
    return (uint16_t)(sgn | ((man + (1u << (shift - 1))) >> shift));
  }
  if (ex >= 31) return (uint16_t)(sgn | 0x7c00u);
  const uint32_t rounded = man + 0x1000u;
  if (rounded & 0x800000u) {
    man = 0;
    if (++ex >= 31) return (uint16_t)(sgn | 0x7c00u);
  } else {
    man = rounded;
  }
  return (uint16_t)(sgn | ((uint32_t)ex << 10) | (man >> 13));
}

void op_to_f16(const float* in, uint16_t* out, int n) {
  for (int i = 0; i < n; ++i) out[i] = op_f2h(in[i]);
}

/* h2f (objprob.cpp:31-47) */
float op_h2f(uint16_t h) {
  const uint32_t sgn = (uint32_t)(h & 0x8000u) << 16;
  uint32_t ex = (h >> 10) & 0x1fu, man = h & 0x3ffu, x;
  if (ex == 0) {
    if (man == 0) {
      x = sgn;
    } else {
      ex = 113;
      while (!(man & 0x400u)) { man <<= 1; --ex; }
      x = sgn | (ex << 23) | ((man & 0x3ffu) << 13);
    }
  } else if (ex == 31) {
    x = sgn | 0x7f800000u | (man << 13);
  } else {
    x = sgn | ((ex + 112) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

/* voxelKey (cloud.cpp:66-69): 21-bit signed-offset cell index per axis, float product */
static uint64_t vq(float v, float inv) { return (uint64_t)((int64_t)floorf(v * inv) + (1 << 20)) & 0x1FFFFFull; }
uint64_t op_voxel_key(float x, float y, float z, float inv) { return vq(x, inv) | vq(y, inv) << 21 | vq(z, inv) << 42; }

/* cellKey3 (objprob.cpp:92-95) */
static uint64_t ck3(int64_t i, int64_t j, int64_t k) {
  return ((uint64_t)(i + (1 << 20)) & 0x1FFFFFull) | ((uint64_t)(j + (1 << 20)) & 0x1FFFFFull) << 21 |
         ((uint64_t)(k + (1 << 20)) & 0x1FFFFFull) << 42;
}

static int cmp_u64(const void* a, const void* b) {
  const uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
  return x < y ? -1 : x > y;
}

/* apBuildContact + apContact (objprob.cpp:470-504): fraction of pts whose 27-neighbourhood of
 * `cell` cells holds a cell of `cloud`; the cell index range of the cloud is the early-out box */
double op_contact(const float* cloud, int nc, const float* pts, int np, double cell) {
  if (np <= 0 || nc <= 0) return 0.0;
  const double inv = 1.0 / cell;
  uint64_t* keys = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)nc);
  int64_t lo[3] = {INT64_MAX, INT64_MAX, INT64_MAX}, hi[3] = {INT64_MIN, INT64_MIN, INT64_MIN};
  for (int i = 0; i < nc; ++i) {
    int64_t c[3];
    for (int k = 0; k < 3; ++k) {
      c[k] = (int64_t)floor(cloud[3 * i + k] * inv);
      if (c[k] < lo[k]) lo[k] = c[k];
      if (c[k] > hi[k]) hi[k] = c[k];
    }
    keys[i] = ck3(c[0], c[1], c[2]);
  }
  qsort(keys, (size_t)nc, sizeof(uint64_t), cmp_u64);
  int nu = 0;
  for (int i = 0; i < nc; ++i)
    if (nu == 0 || keys[nu - 1] != keys[i]) keys[nu++] = keys[i];
  int hit = 0;
  for (int i = 0; i < np; ++i) {
    const int64_t a = (int64_t)floor(pts[3 * i] * inv), b = (int64_t)floor(pts[3 * i + 1] * inv),
                  c = (int64_t)floor(pts[3 * i + 2] * inv);
    if (a < lo[0] - 1 || a > hi[0] + 1 || b < lo[1] - 1 || b > hi[1] + 1 || c < lo[2] - 1 || c > hi[2] + 1) continue;
    int found = 0;
    for (int dx = -1; dx <= 1 && !found; ++dx)
      for (int dy = -1; dy <= 1 && !found; ++dy)
        for (int dz = -1; dz <= 1 && !found; ++dz) {
          const uint64_t key = ck3(a + dx, b + dy, c + dz);
          found = bsearch(&key, keys, (size_t)nu, sizeof(uint64_t), cmp_u64) != NULL;
        }
    hit += found;
  }
  free(keys);
  return (double)hit / np;
}

/* eigSym3 (objprob.cpp:50-84): cyclic-by-largest Jacobi rotations, <= 32 sweeps, eigenvalues
 * ascending (ties keep index order), eigenvectors as columns of V */
void op_eig_sym3(double A[3][3], double ev[3], double V[3][3]) {
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) V[i][j] = i == j;
  for (int sweep = 0; sweep < 32; ++sweep) {
    int p = 0, q = 1;
    double big = fabs(A[0][1]);
    if (fabs(A[0][2]) > big) { big = fabs(A[0][2]); p = 0; q = 2; }
    if (fabs(A[1][2]) > big) { big = fabs(A[1][2]); p = 1; q = 2; }
    if (big < 1e-12) break;
    const double th = 0.5 * atan2(2 * A[p][q], A[q][q] - A[p][p]);
    const double c = cos(th), s = sin(th);
    for (int k = 0; k < 3; ++k) {
      const double u = A[k][p], w = A[k][q];
      A[k][p] = c * u - s * w;
      A[k][q] = s * u + c * w;
    }
    for (int k = 0; k < 3; ++k) {
      const double u = A[p][k], w = A[q][k];
      A[p][k] = c * u - s * w;
      A[q][k] = s * u + c * w;
    }
    for (int k = 0; k < 3; ++k) {
      const double u = V[k][p], w = V[k][q];
      V[k][p] = c * u - s * w;
      V[k][q] = s * u + c * w;
    }
  }
  int o[3] = {0, 1, 2};
  for (int i = 1; i < 3; ++i)
    for (int j = i; j > 0 && A[o[j]][o[j]] < A[o[j - 1]][o[j - 1]]; --j) {
      const int t = o[j];
      o[j] = o[j - 1];
      o[j - 1] = t;
    }
  double W[3][3];
  for (int k = 0; k < 3; ++k) {
    ev[k] = A[o[k]][o[k]];
    for (int i = 0; i < 3; ++i) W[i][k] = V[i][o[k]];
  }
  memcpy(V, W, sizeof W);
}

static int cmp_d(const void* a, const void* b) {
  const double x = *(const double*)a, y = *(const double*)b;
  return x < y ? -1 : x > y;
}

/* pctOf (objprob.cpp:86-90): the value std::nth_element leaves at k = min(n-1, q(n-1)+0.5),
 * i.e. the k-th order statistic (sorts v in place) */
static double pct_of(double* v, int n, double q) {
  size_t k = (size_t)(q * (double)(n - 1) + 0.5);
  if (k > (size_t)(n - 1)) k = (size_t)(n - 1);
  qsort(v, (size_t)n, sizeof(double), cmp_d);
  return v[k];
}

/* pcaOf (objprob.cpp:101-114): sequential mean and covariance of the listed points */
static void pca_of(const float* xyz, const int* idx, int ni, double m[3], double ev[3], double V[3][3]) {
  m[0] = m[1] = m[2] = 0;
  for (int t = 0; t < ni; ++t)
    for (int k = 0; k < 3; ++k) m[k] += xyz[3 * idx[t] + k];
  const double inv = 1.0 / (double)(ni > 1 ? ni : 1);
  for (int k = 0; k < 3; ++k) m[k] *= inv;
  double C[3][3] = {{0, 0, 0}, {0, 0, 0}, {0, 0, 0}};
  for (int t = 0; t < ni; ++t) {
    const int i = idx[t];
    const double d[3] = {xyz[3 * i] - m[0], xyz[3 * i + 1] - m[1], xyz[3 * i + 2] - m[2]};
    for (int a = 0; a < 3; ++a)
      for (int b = 0; b < 3; ++b) C[a][b] += d[a] * d[b];
  }
  for (int a = 0; a < 3; ++a)
    for (int b = 0; b < 3; ++b) C[a][b] *= inv;
  op_eig_sym3(C, ev, V);
}

/* apPlaneFit (objprob.cpp:130-209).  out[10] = ok, n0, n1, n2, thick, inl, zmed, zlo, zhi,
 * hspan; the reference's ApPlane defaults when no plane is found (objprob.hpp:198-203).
 * 1. RANSAC over a <= 256-point subsample at stride max(1, n/min(n,256)), hypotheses from
 *    three distinct splitmix-drawn indices, adaptive stop (99 % confidence on w^3);
 * 2. two PCA refits on the inliers of the current plane;
 * 3. thickness, inlier ratio, 10/50/90 % z and 10-90 % horizontal spread of the inliers. */
int op_plane_fit(const float* xyz, int n, double tau, uint64_t seed, int max_iters, double* out) {
  const double dflt[10] = {0, 0, 0, 1, 1, 0, 0, 0, 0, 0};
  memcpy(out, dflt, sizeof dflt);
  if (n < 8 || tau <= 0) return 0;
  uint64_t rs = seed ^ ((uint64_t)n << 32);
  const int ns = n < 256 ? n : 256;
  const int sstep = n / ns > 1 ? n / ns : 1;
  double best[4] = {0, 0, 1, 0};
  int best_c = -1, need = max_iters > 1 ? max_iters : 1;
  for (int it = 0; it < need && it < max_iters; ++it) {
    int i0, i1, i2;
    i0 = (int)(sm_next(&rs) % (uint64_t)n);
    do i1 = (int)(sm_next(&rs) % (uint64_t)n); while (i1 == i0);
    do i2 = (int)(sm_next(&rs) % (uint64_t)n); while (i2 == i0 || i2 == i1);
    const float *a = xyz + 3 * i0, *b = xyz + 3 * i1, *c = xyz + 3 * i2;
    const double u[3] = {b[0] - a[0], b[1] - a[1], b[2] - a[2]}, v[3] = {c[0] - a[0], c[1] - a[1], c[2] - a[2]};
    double nn[3] = {u[1] * v[2] - u[2] * v[1], u[2] * v[0] - u[0] * v[2], u[0] * v[1] - u[1] * v[0]};
    const double L = sqrt(nn[0] * nn[0] + nn[1] * nn[1] + nn[2] * nn[2]);
    if (L < 1e-6) continue;
    for (int k = 0; k < 3; ++k) nn[k] /= L;
    const double d0 = -(nn[0] * a[0] + nn[1] * a[1] + nn[2] * a[2]);
    int cnt = 0;
    for (int i = 0; i < n; i += sstep) cnt += fabs(nn[0] * xyz[3 * i] + nn[1] * xyz[3 * i + 1] + nn[2] * xyz[3 * i + 2] + d0) <= tau;
    if (cnt > best_c) {
      best_c = cnt;
      best[0] = nn[0]; best[1] = nn[1]; best[2] = nn[2]; best[3] = d0;
      const double w = (double)cnt / (double)((n + sstep - 1) / sstep);
      const double pw = w * w * w;
      if (pw > 0.999999) break;
      if (pw > 1e-9) {
        const int k = (int)ceil(log(0.01) / log(1.0 - pw));
        need = k > 8 ? k : 8;
      }
    }
  }
  if (best_c < 3) return 0;
  int* in = (int*)malloc(sizeof(int) * (size_t)n);
  int ni = 0;
  double m[3], ev[3], V[3][3], ref[4];
  const double* pl = best;
  for (int pass = 0; pass < 2; ++pass) {
    ni = 0;
    for (int i = 0; i < n; ++i)
      if (fabs(pl[0] * xyz[3 * i] + pl[1] * xyz[3 * i + 1] + pl[2] * xyz[3 * i + 2] + pl[3]) <= tau) in[ni++] = i;
    if (ni < 3) { free(in); return 0; }
    pca_of(xyz, in, ni, m, ev, V);
    ref[0] = V[0][0]; ref[1] = V[1][0]; ref[2] = V[2][0];
    ref[3] = -(ref[0] * m[0] + ref[1] * m[1] + ref[2] * m[2]);
    pl = ref;
  }
  double sxx = 0, sxy = 0, syy = 0;
  for (int t = 0; t < ni; ++t) {
    const double dx = xyz[3 * in[t]] - m[0], dy = xyz[3 * in[t] + 1] - m[1];
    sxx += dx * dx; sxy += dx * dy; syy += dy * dy;
  }
  const double th = 0.5 * atan2(2 * sxy, sxx - syy), hc = cos(th), hs = sin(th);
  double* z = (double*)malloc(sizeof(double) * (size_t)ni);
  double* h = (double*)malloc(sizeof(double) * (size_t)ni);
  for (int t = 0; t < ni; ++t) {
    const int i = in[t];
    const double d0 = xyz[3 * i] - m[0], d1 = xyz[3 * i + 1] - m[1];
    z[t] = xyz[3 * i + 2];
    h[t] = d0 * hc + d1 * hs;
  }
  out[0] = 1;
  out[1] = V[0][0]; out[2] = V[1][0]; out[3] = V[2][0];
  out[4] = sqrt(ev[0] > 0.0 ? ev[0] : 0.0);
  out[5] = (double)ni / n;
  const double h9 = pct_of(h, ni, 0.9), h1 = pct_of(h, ni, 0.1);
  out[9] = h9 - h1;
  out[7] = pct_of(z, ni, 0.1);
  out[8] = pct_of(z, ni, 0.9);
  out[6] = pct_of(z, ni, 0.5);
  free(z); free(h); free(in);
  return 1;
}

/* fastAtan2 (scan.cpp:19-30): the reference's float polynomial arctangent, restated as is */
float op_fast_atan2(float y, float x) {
  const float ax = fabsf(x), ay = fabsf(y);
  const float mx = fmaxf(ax, ay), mn = fminf(ax, ay);
  if (mx == 0.f) return 0.f;
  const float t = mn / mx, s = t * t;
  float r = ((((-0.0117212f * s + 0.05265332f) * s - 0.11643287f) * s + 0.19354346f) * s - 0.33262347f) * s + 0.99997726f;
  r *= t;
  if (ay > ax) r = 1.57079637f - r;
  if (x < 0) r = 3.14159274f - r;
  return y < 0 ? -r : r;
}
