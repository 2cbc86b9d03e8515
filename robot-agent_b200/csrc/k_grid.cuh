// 2D occupancy of a keyframe: makeScan (scenemap src/scan.cpp:222-451), the Mapper2D insert
// policy (mapper2d.cpp:46-72) and OccGrid::insert (grid.cpp:95-159).  One CTA per map.
//
// makeScan: per-pixel base-frame points at stride `step`; per-bin nearest in-band hit = the
// first raster pixel with the smallest squared range (64-bit atomicMin of (rr2 bits, pixel));
// floor rays = max squared range; dense match points accumulate per 2.5 cm cell in raster order
// (cells ranked by their first pixel; each cell's pixels summed in raster order by one thread).
// OccGrid::insert: one update per cell per scan, hits before misses, and the first hit of a cell
// feeds its point sums.  Made parallel with a per-cell first-touch key (scan id, order): hit
// points carry their sequence order, ray cells carry a miss order above every hit, and only the
// occurrence holding the minimum key applies the update.
#pragma once
#include "k_merge.cuh"

#define GRID_THREADS 1024
#define MH_SLOTS 16384

// fastAtan2 polynomial of the reference (scenemap scan.cpp:140-151), float, no FMA contraction
DEV float fast_atan2(float y, float x) {
  const float ax = fabsf(x), ay = fabsf(y);
  const float mx = fmaxf(ax, ay), mn = fminf(ax, ay);
  if (mx == 0.f) return 0.f;
  const float a = mn / mx, s = a * a;
  float r = ((((-0.0117212f * s + 0.05265332f) * s - 0.11643287f) * s + 0.19354346f) * s - 0.33262347f) * s + 0.99997726f;
  r *= a;
  if (ay > ax) r = 1.57079637f - r;
  if (x < 0) r = 3.14159274f - r;
  return y < 0 ? -r : r;
}

DEV float fdist2(float ax, float ay, float az, const float* b) {
  const float dx = ax - b[0], dy = ay - b[1], dz = az - b[2];
  return dx * dx + dy * dy + dz * dz;
}

DEV int cell_of(double v, float res) { return (int)floor(v / (double)res); }

__global__ void __launch_bounds__(GRID_THREADS) k_grid(Batch B) {
  __shared__ BlockScratch bs;
  __shared__ int sh_n[4];
  __shared__ int sh_ins;
  __shared__ int sh_c8;   // a visible (export8) value changed in this insert (cells_changed_)
  const int m = B.map0 + blockIdx.x, tid = threadIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active) return;
  MapRec* R = &B.maps[m];
  const smg_params& P = B.p;
  const float* T = F.T_bc;
  const int step = max(1, (int)llround(F.w / 160.0));
  const int gw = (F.w + step - 1) / step, gh = (F.h + step - 1) / step, ng = gw * gh;
  if (ng > B.scan_pmax) {
    if (tid == 0) { set_err(R, SMG_E_CAP_GRID); R->kf_inserted = 0; R->kf_changed = 0; }
    return;
  }
  float4* SP = B.sP + (size_t)m * B.scan_pmax;
  const int nb = P.bins;
  unsigned long long* HK = B.hit_key + (size_t)m * nb;
  float* FR = B.floor_r + (size_t)m * nb;
  int16_t* SIG = B.sig + (size_t)m * nb;
  int64_t* MK = B.mkey + (size_t)m * B.scan_pmax;
  float4* MV = B.mval + (size_t)m * B.scan_pmax;
  PHASE_START();
  // 1. base-frame points (scan.cpp:233-251)
  const float ifx = 1.f / F.fx;
  for (int c = tid; c < ng; c += blockDim.x) {
    const int j = c / gw, i = c - j * gw;
    const int v = j * step, u = i * step;
    const float z = F.depth[(size_t)v * F.w + u];
    float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
    if (z >= P.scan_zmin && z <= P.scan_zmax) {
      const float yn = ((float)v - F.cy) / F.fy;
      const float ry0 = T[1] * yn + T[2], ry1 = T[5] * yn + T[6], ry2 = T[9] * yn + T[10];
      const float xn = ((float)u - F.cx) * ifx;
      q.x = (T[0] * xn + ry0) * z + T[3];
      q.y = (T[4] * xn + ry1) * z + T[7];
      q.z = (T[8] * xn + ry2) * z + T[11];
      q.w = z;
    }
    SP[c] = q;
  }
  for (int k = tid; k < nb; k += blockDim.x) { HK[k] = ~0ull; FR[k] = 0.f; }
  __syncthreads();
  PHASE_MARK(24);   // base-frame points
  // 2. classification (scan.cpp:254-416)
  const float bsc = (float)nb / (2.f * 3.14159274f);
  float ab[2][3], ab2[2];
  for (int s = 0; s < 2; ++s) {
    for (int k = 0; k < 3; ++k) ab[s][k] = F.eef_base[s][k] - P.shoulder[s][k];
    ab2[s] = fmaxf(ab[s][0] * ab[s][0] + ab[s][1] * ab[s][1] + ab[s][2] * ab[s][2], 1e-9f);
  }
  const float self2 = P.self_r * P.self_r, eef2 = P.eef_r * P.eef_r, arm2 = P.arm_r * P.arm_r;
  const float inv_mc = 1.f / P.match_cell;
  for (int c = tid; c < ng; c += blockDim.x) {
    MK[c] = INT64_MIN;
    const float4 q = SP[c];
    if (q.w == 0.f) continue;
    const float px = q.x, py = q.y, pz = q.z;
    const float r2 = px * px + py * py;
    if (r2 < self2) continue;
    bool self = false;
    for (int s = 0; s < 2 && !self; ++s) {
      if (fdist2(px, py, pz, F.eef_base[s]) < eef2) { self = true; break; }
      const float* a = P.shoulder[s];
      float t = ((px - a[0]) * ab[s][0] + (py - a[1]) * ab[s][1] + (pz - a[2]) * ab[s][2]) / ab2[s];
      t = fminf(fmaxf(t, 0.f), 1.f);
      const float cc[3] = {a[0] + t * ab[s][0], a[1] + t * ab[s][1], a[2] + t * ab[s][2]};
      if (fdist2(px, py, pz, cc) < arm2) self = true;
    }
    if (self) continue;
    const int j = c / gw, i = c - j * gw;
    if (pz <= P.band_hi) {
      const float yn = ((float)(j * step) - F.cy) / F.fy;
      const float xn = ((float)(i * step) - F.cx) * ifx;
      const float a = T[0] * xn + T[1] * yn + T[2], bq = T[4] * xn + T[5] * yn + T[6];
      int k = (int)((fast_atan2(bq, a) + 3.14159274f) * bsc);
      k = k < 0 ? 0 : (k >= nb ? nb - 1 : k);
      const float zz = q.w;
      const float rr2 = zz * zz * (a * a + bq * bq);
      if (pz < P.band_lo) atomicMax((unsigned int*)&FR[k], __float_as_uint(rr2));
      else atomicMin(&HK[k], ((unsigned long long)__float_as_uint(rr2) << 32) | (unsigned int)c);
    }
    if (!P.dense || pz < P.band_lo || pz > P.match_hi || i == 0 || j == 0 || i == gw - 1 || j == gh - 1) continue;
    const float4 L = SP[c - 1], Rr = SP[c + 1], U = SP[c - gw], Dn = SP[c + gw];
    if (L.w == 0.f || Rr.w == 0.f || U.w == 0.f || Dn.w == 0.f) continue;
    const float z = q.w;
    if (fabsf(Rr.w - L.w) >= 0.1f * z || fabsf(Dn.w - U.w) >= 0.1f * z) continue;
    const float ax = Rr.x - L.x, ay = Rr.y - L.y, az = Rr.z - L.z;
    const float bx = Dn.x - U.x, by = Dn.y - U.y, bz = Dn.z - U.z;
    const float nx = ay * bz - az * by, ny = az * bx - ax * bz, nz = ax * by - ay * bx;
    const float nn2 = nx * nx + ny * ny + nz * nz;
    const float vz = P.vert_nz;
    if (nn2 <= 0 || nz * nz >= vz * vz * nn2) continue;
    const int64_t key = (int64_t)(((unsigned long long)(long long)floorf(px * inv_mc) << 32) ^
                                  ((unsigned long long)(long long)floorf(py * inv_mc) & 0xffffffffull));
    const float hn = sqrtf(nx * nx + ny * ny);
    float ux = nx / hn, uy = ny / hn;
    if (ux * (T[3] - px) + uy * (T[7] - py) < 0) { ux = -ux; uy = -uy; }
    MK[c] = key;
    MV[c] = make_float4(px, py, ux, uy);
  }
  __syncthreads();
  PHASE_MARK(25);   // classification
  // 3. match cells: first pixel per key, rank by first pixel, per-cell raster-order sums
  int64_t* HKY = B.mh_key + (size_t)m * MH_SLOTS;
  int32_t* HF = B.mh_first + (size_t)m * MH_SLOTS;
  int32_t* HC = B.mh_cell + (size_t)m * MH_SLOTS;
  int32_t* CF = B.mcell_first + (size_t)m * B.scan_pmax;   // per pixel: 1 if first pixel of a cell
  int32_t* CC = B.mcell_cnt + (size_t)m * B.scan_pmax;     // per rank
  int32_t* CO = B.mcell_off + (size_t)m * B.scan_pmax;     // per rank: bucket offset, then fill
  int32_t* CPX = B.mcell_pix + (size_t)m * B.scan_pmax;    // bucketed pixels
  for (int i = tid; i < MH_SLOTS; i += blockDim.x) { HKY[i] = INT64_MIN; HF[i] = 0x7fffffff; }
  for (int c = tid; c < ng; c += blockDim.x) CF[c] = 0;
  __syncthreads();
  PHASE_MARK(30);
  for (int c = tid; c < ng; c += blockDim.x) {
    const int64_t key = MK[c];
    if (key == INT64_MIN) continue;
    uint32_t h = (uint32_t)(((uint64_t)key * 0x9E3779B97F4A7C15ull) >> 50) & (MH_SLOTS - 1);
    for (int probe = 0; probe < MH_SLOTS; ++probe) {
      const unsigned long long prev = atomicCAS((unsigned long long*)&HKY[h], (unsigned long long)INT64_MIN, (unsigned long long)key);
      if (prev == (unsigned long long)INT64_MIN || prev == (unsigned long long)key) { atomicMin(&HF[h], c); break; }
      h = (h + 1) & (MH_SLOTS - 1);
    }
  }
  __syncthreads();
  PHASE_MARK(31);
  for (int i = tid; i < MH_SLOTS; i += blockDim.x)
    if (HKY[i] != INT64_MIN && INB(HF[i], ng, 702)) CF[HF[i]] = 1;
  __syncthreads();
  PHASE_MARK(32);
  // rank of each cell = number of cells whose first pixel comes earlier (ordered scan)
  int nrank = 0;
  for (int c0 = 0; c0 < ng; c0 += blockDim.x) {
    const int c = c0 + tid;
    const int f = c < ng ? CF[c] : 0;
    int tot;
    const int pos = block_excl_scan(f, &tot, bs);
    if (f) CF[c] = 1 + nrank + pos;   // rank + 1
    nrank += tot;
  }
  __syncthreads();
  PHASE_MARK(33);
  const int ncell = nrank < SMG_MATCH_CELLS ? nrank : SMG_MATCH_CELLS;   // later cells are dropped
  for (int i = tid; i < MH_SLOTS; i += blockDim.x)
    if (HKY[i] != INT64_MIN) HC[i] = CF[HF[i]] - 1;
  for (int r = tid; r < ncell; r += blockDim.x) CC[r] = 0;
  __syncthreads();
  // per-pixel cell rank -> counts
  for (int c = tid; c < ng; c += blockDim.x) {
    const int64_t key = MK[c];
    if (key == INT64_MIN) continue;
    uint32_t h = (uint32_t)(((uint64_t)key * 0x9E3779B97F4A7C15ull) >> 50) & (MH_SLOTS - 1);
    for (int probe = 0; probe < MH_SLOTS && HKY[h] != key; ++probe) h = (h + 1) & (MH_SLOTS - 1);
    if (HKY[h] != key) { set_err(R, SMG_E_CAP_GRID); MK[c] = -1; continue; }
    const int r = HC[h];
    MK[c] = r < ncell ? r : -1;   // reuse: rank or -1
    if (r < ncell) atomicAdd(&CC[r], 1);
  }
  __syncthreads();
  PHASE_MARK(34);
  int off = 0;
  for (int r0 = 0; r0 < ncell; r0 += blockDim.x) {
    const int r = r0 + tid;
    const int v = r < ncell ? CC[r] : 0;
    int tot;
    const int pos = block_excl_scan(v, &tot, bs);
    if (r < ncell) CO[r] = off + pos;
    off += tot;
  }
  __syncthreads();
  for (int c = tid; c < ng; c += blockDim.x) {
    const long long r = MK[c];
    if (r < 0 || MK[c] == INT64_MIN) continue;
    const int slot = atomicAdd(&CO[r], 1);
    if (INB(slot, ng, 701)) CPX[slot] = c;
  }
  __syncthreads();
  PHASE_MARK(35);
  // raster order within each cell: a bucketed pixel's place is the number of pixels of its
  // cell with a smaller index (every slot counts over its own bucket, in parallel)
  int32_t* SPX = CF;   // the per-pixel first flags are dead here: sorted buckets
  for (int a = tid; a < off; a += blockDim.x) {
    const int v = CPX[a];
    const long long r = MK[v];
    if (r < 0 || r >= ncell) continue;
    const int e = CO[r], s0 = e - CC[r];
    int pos = 0;
    for (int b = s0; b < e; ++b) pos += CPX[b] < v;
    if (INB(s0 + pos, ng, 706)) SPX[s0 + pos] = v;
  }
  __syncthreads();
  PHASE_MARK(36);
  float* OUT = B.sc_pts + (size_t)m * (2 * SMG_BINS_MAX + SMG_MATCH_CELLS) * 4;
  for (int r = tid; r < ncell; r += blockDim.x) {
    const int n = CC[r], e = CO[r], s0 = e - n;
    float sx = 0, sy = 0, snx = 0, sny = 0;
    int a = s0;
    for (; a + 4 <= e; a += 4) {   // four loads in flight, added in order
      const float4 w0 = MV[SPX[a]], w1 = MV[SPX[a + 1]], w2 = MV[SPX[a + 2]], w3 = MV[SPX[a + 3]];
      sx += w0.x; sy += w0.y; snx += w0.z; sny += w0.w;
      sx += w1.x; sy += w1.y; snx += w1.z; sny += w1.w;
      sx += w2.x; sy += w2.y; snx += w2.z; sny += w2.w;
      sx += w3.x; sy += w3.y; snx += w3.z; sny += w3.w;
    }
    for (; a < e; ++a) {
      const float4 w = MV[SPX[a]];
      sx += w.x; sy += w.y; snx += w.z; sny += w.w;
    }
    const float nn = sqrtf(snx * snx + sny * sny);
    OUT[4 * r] = sx / n;
    OUT[4 * r + 1] = sy / n;
    OUT[4 * r + 2] = nn > 1e-6f ? snx / nn : 0.f;
    OUT[4 * r + 3] = nn > 1e-6f ? sny / nn : 0.f;
  }
  __syncthreads();
  PHASE_MARK(26);   // match cells
  // 4. laser line and free rays in bin order; signature (scan.cpp:427-440)
  const float isc = 1.f / P.grid_res;
  float* HOUT = OUT + 4 * SMG_MATCH_CELLS;
  float* FOUT = HOUT + 4 * SMG_BINS_MAX;
  int nh = 0, nf = 0;
  for (int k0 = 0; k0 < nb; k0 += blockDim.x) {
    const int k = k0 + tid;
    int ish = 0, isf = 0;
    float hr = 0, fr = 0;
    int pix = -1;
    if (k < nb) {
      const unsigned long long hk = HK[k];
      if (hk != ~0ull) { ish = 1; hr = sqrtf(__uint_as_float((unsigned)(hk >> 32))); pix = (int)(hk & 0xffffffffu); }
      else if (FR[k] > 0) { isf = 1; fr = sqrtf(FR[k]); }
      SIG[k] = ish ? (int16_t)fminf(32000.f, hr * isc + 1.f) : (isf ? (int16_t)(-fminf(32000.f, fr * isc + 1.f)) : 0);
    }
    int th, tf;
    const int ph = block_excl_scan(ish, &th, bs);
    const int pf = block_excl_scan(isf, &tf, bs);
    if (ish && INB(pix, ng, 705)) { const float4 q = SP[pix]; HOUT[4 * (nh + ph)] = q.x; HOUT[4 * (nh + ph) + 1] = q.y; }
    if (isf) {
      FOUT[4 * (nf + pf)] = T[3] + fr * B.bin_cos[k];
      FOUT[4 * (nf + pf) + 1] = T[7] + fr * B.bin_sin[k];
    }
    nh += th;
    nf += tf;
  }
  __syncthreads();
  PHASE_MARK(27);   // laser line, free rays, signature
  // 5. insert policy (mapper2d.cpp:46-72)
  const int th_c = P.change_cells;
  int nd_l = 0;
  const int16_t* IS = B.ins_sig + (size_t)m * nb;
  for (int k = tid; k < nb; k += blockDim.x) {
    const int dlt = (int)IS[k] - (int)SIG[k];
    nd_l += (dlt > th_c || dlt < -th_c || ((IS[k] > 0) != (SIG[k] > 0)));
  }
  const int nd_s = block_sum_i(nd_l, bs);
  if (tid == 0) {
    ++R->kf_since;
    const int nd = R->kf_sig_n == nb ? nd_s : (1 << 20);
    const bool changed = nd > P.change_bins;
    double da = F.base[2] - R->kf_last_ins[2];
    da = fmod(da + 3.141592653589793, 2 * 3.141592653589793);
    if (da < 0) da += 2 * 3.141592653589793;
    da -= 3.141592653589793;
    const bool nudged = hypot(F.base[0] - R->kf_last_ins[0], F.base[1] - R->kf_last_ins[1]) >= 0.01 ||
                        fabs(da) >= 0.5 * 3.141592653589793 / 180.0;
    sh_ins = R->kf_first || nudged || changed || R->kf_last_changed > 0 || R->kf_since >= P.still_every;
    R->kf_hits = P.dense ? ncell : nh;
    R->kf_inserted = sh_ins;
    if (!sh_ins) R->kf_changed = 0;
    sh_n[0] = ncell; sh_n[1] = nh; sh_n[2] = nf;
  }
  __syncthreads();
  PHASE_MARK(28);   // insert policy
  if (!sh_ins) return;
  // 6. OccGrid::insert (grid.cpp:95-159)
  const double c = F.cos_th, sn = F.sin_th;
  const double* pose = F.base;
  const float res = P.grid_res;
  const double ox = pose[0] + c * (double)T[3] - sn * (double)T[7], oy = pose[1] + sn * (double)T[3] + c * (double)T[7];
  const int cx = cell_of(ox, res), cy = cell_of(oy, res);
  const int nm = sh_n[0], nhh = sh_n[1], nff = sh_n[2], npt = nm + nhh + nff;
  const int GW = B.gw_grid, GH = B.gh_grid, X0 = B.gx0, Y0 = B.gy0;
  const size_t gbase = (size_t)m * GW * GH;
  unsigned long long* TOUCH = B.gtouch + gbase;
  if (tid == 0) { ++R->scan_id; wk_add(R, SMG_WK_SCAN_PX, ng); wk_add(R, SMG_WK_SCAN_PTS, npt); }
  __syncthreads();
  const unsigned long long sk = (unsigned long long)(0xffffffffu - R->scan_id) << 32;
  int bad = 0;
  bad |= cx < X0 || cy < Y0 || cx >= X0 + GW || cy >= Y0 + GH;
  // point k -> (ix, iy, wx, wy)
  auto pt_of = [&](int k, float* x, float* y) {
    const float* src = k < nm ? OUT + 4 * k : (k < nm + nhh ? HOUT + 4 * (k - nm) : FOUT + 4 * (k - nm - nhh));
    *x = src[0];
    *y = src[1];
  };
  for (int k = tid; k < npt; k += blockDim.x) {
    float x, y;
    pt_of(k, &x, &y);
    const double wx = pose[0] + c * (double)x - sn * (double)y, wy = pose[1] + sn * (double)x + c * (double)y;
    const int ix = cell_of(wx, res), iy = cell_of(wy, res);
    if (ix < X0 || iy < Y0 || ix >= X0 + GW || iy >= Y0 + GH) { bad = 1; continue; }
    if (k < nm + nhh) atomicMin(&TOUCH[(size_t)(iy - Y0) * GW + (ix - X0)], sk | (unsigned)k);
  }
  bad = block_sum_i(bad, bs);
  if (bad) {
    if (tid == 0) set_err(R, SMG_E_CAP_GRID);
    return;
  }
  // rays: laser hits (end excluded), free rays (end included) — Bresenham (grid.cpp:236-256)
  const int nray = nhh + nff;
  int applied_l = 0;
  if (tid == 0) sh_c8 = 0;
  for (int pass = 0; pass < 2; ++pass) {
    int changed_l = 0;
    for (int r = tid; r < nray; r += blockDim.x) {
      float x, y;
      pt_of(nm + r, &x, &y);
      const double wx = pose[0] + c * (double)x - sn * (double)y, wy = pose[1] + sn * (double)x + c * (double)y;
      const int x1 = cell_of(wx, res), y1 = cell_of(wy, res);
      int xx = cx, yy = cy;
      const int dx = abs(x1 - xx), dy = -abs(y1 - yy), sx = xx < x1 ? 1 : -1, sy = yy < y1 ? 1 : -1;
      int err = dx + dy;
      unsigned stepi = 0;
      const bool is_free = r >= nhh;
      for (;;) {
        const bool end = xx == x1 && yy == y1;
        if (end && !is_free) break;
        if (!INB(xx - X0, GW, 703) || !INB(yy - Y0, GH, 704)) break;
        const size_t ci = (size_t)(yy - Y0) * GW + (xx - X0);
        const unsigned long long key = sk | 0x80000000ull | ((unsigned long long)r << 12) | (stepi & 0xfffu);
        if (pass == 0) {
          atomicMin(&TOUCH[ci], key);
        } else if (TOUCH[ci] == key) {   // miss (grid.cpp:175-193)
          int16_t* Lp = B.gL + gbase + ci;
          uint8_t* fl = B.gflags + gbase + ci;
          const int16_t L = *Lp;
          const int nL = max((int)L + B.q_miss, (int)B.q_min);
          const bool was_seen = *fl & 1;
          *fl |= 1;
          ++applied_l;
          if (!(nL == L && was_seen)) {
            ++changed_l;
            *Lp = (int16_t)nL;
            const int8_t c8 = B.lut8[nL + B.lut_off];
            if (B.gc8[gbase + ci] != c8) sh_c8 = 1;
            B.gc8[gbase + ci] = c8;
            if (nL <= 0 && (*fl & 2)) {
              *fl &= (uint8_t)~2u;
              B.gcold[gbase + ci] = make_float4(0.f, 0.f, 0.f, 0.f);
              B.gcnt[gbase + ci] = 0;
            }
          }
        }
        if (end) break;
        ++stepi;
        const int e2 = 2 * err;
        if (e2 >= dy) { err += dy; xx += sx; }
        if (e2 <= dx) { err += dx; yy += sy; }
      }
    }
    if (pass == 0) {
      __syncthreads();
      // hits (grid.cpp:157-173, 224-234): the point holding the cell's minimum key applies it
      for (int k = tid; k < nm + nhh; k += blockDim.x) {
        float x, y;
        pt_of(k, &x, &y);
        const double wx = pose[0] + c * (double)x - sn * (double)y, wy = pose[1] + sn * (double)x + c * (double)y;
        const int ix = cell_of(wx, res), iy = cell_of(wy, res);
        const size_t ci = (size_t)(iy - Y0) * GW + (ix - X0);
        if (TOUCH[ci] != (sk | (unsigned)k)) continue;
        float nx = 0.f, ny = 0.f;
        if (k < nm) {
          const float mnx = OUT[4 * k + 2], mny = OUT[4 * k + 3];
          nx = (float)(c * (double)mnx - sn * (double)mny);
          ny = (float)(sn * (double)mnx + c * (double)mny);
        }
        int16_t* Lp = B.gL + gbase + ci;
        uint8_t* fl = B.gflags + gbase + ci;
        const int16_t L = *Lp;
        ++applied_l;
        const int nL = min((int)L + B.q_hit, (int)B.q_max);
        const bool was_seen = *fl & 1;
        *fl |= 3;
        changed_l += (nL != L) | !was_seen;
        *Lp = (int16_t)nL;
        const int8_t c8 = B.lut8[nL + B.lut_off];
        if (B.gc8[gbase + ci] != c8) sh_c8 = 1;
        B.gc8[gbase + ci] = c8;
        float4 cold = B.gcold[gbase + ci];
        uint32_t cnt = B.gcnt[gbase + ci];
        uint32_t c1 = cnt & 0xffffu, c2 = cnt >> 16;
        if (c1 < 60000) { cold.x += (float)wx; cold.y += (float)wy; ++c1; }
        if ((nx != 0 || ny != 0) && c2 < 60000) { cold.z += nx; cold.w += ny; ++c2; }
        B.gcold[gbase + ci] = cold;
        B.gcnt[gbase + ci] = c1 | c2 << 16;
      }
      __syncthreads();
    }
    const int ch = block_sum_i(changed_l, bs);
    if (tid == 0) {
      if (pass == 0) sh_n[3] = ch;
      else {
        R->kf_changed = sh_n[3] + ch;
        R->kf_last_changed = R->kf_changed;
        if (sh_c8) R->w_dirty = 1;   // the wall extraction's grid_changed (cellsVersion)
        R->kf_last_ins[0] = pose[0];
        R->kf_last_ins[1] = pose[1];
        R->kf_last_ins[2] = pose[2];
        R->kf_since = 0;
        R->kf_first = 0;
        R->kf_sig_n = nb;
      }
    }
    __syncthreads();
  }
  applied_l = block_sum_i(applied_l, bs);
  if (tid == 0) wk_add(R, SMG_WK_CELLS, applied_l);
  int16_t* ISw = B.ins_sig + (size_t)m * nb;
  for (int k = tid; k < nb; k += blockDim.x) ISw[k] = SIG[k];
  PHASE_MARK(29);   // insert
}
