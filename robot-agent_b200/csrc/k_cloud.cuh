// Object point clouds: ObjCloud::add (scenemap src/cloud.cpp:86-127) and the contact-cell index
// (apBuildContact, objprob.cpp:470-487), as block-wide device functions.
//
// Cloud slot layout: cpts[2*cap] float4 (x, y, z relative to org, seq as bits), crgb[2*cap]
// (room for the points of one call before the trim), a persistent voxel-key -> index hash
// (generation-tagged, HC >= 2 * 2*cap slots) and the contact-cell set (HCC >= 2*cap slots).
// An add call keeps the reference's sequential semantics: a key new to the cloud is appended at
// its FIRST occurrence in the call, and every voxel keeps the data of the LAST point that hit it.
// The call is parallel: a per-call hash of the call's keys records first/last occurrence, first
// occurrences of new keys are appended by an ordered compaction.
#pragma once
#include "k_update.cuh"

struct CloudCall {
  unsigned long long key;
  uint32_t first, last;
};

// per-CTA work area (global): call hash, keys, destinations, trim buffers
struct Work {
  CloudCall* tab;   // 4 * WORK_N (a call of n <= WORK_N points uses pow2 >= 2n slots)
  uint64_t* keys;   // WORK_N
  int32_t* dst;     // WORK_N
  double* scr;      // WORK_N
  float4* t4;       // WORK_N
  uint32_t* tc;     // WORK_N
};

DEV Work work_at(const Batch& B, int m, int j) {
  unsigned char* w = B.work + ((size_t)m * WORK_SLOTS + j) * B.work_stride;
  Work r;
  const size_t N = (size_t)B.work_n;
  r.tab = (CloudCall*)w;
  r.keys = (uint64_t*)(w + 4 * N * sizeof(CloudCall));
  r.dst = (int32_t*)(r.keys + N);
  r.scr = (double*)(r.dst + N + (N & 1));
  r.t4 = (float4*)(r.scr + N);
  r.tc = (uint32_t*)(r.t4 + N);
  return r;
}

DEV int voxel_lookup(const Batch& B, size_t cs, uint32_t gen, uint64_t key) {
  const uint64_t* K = B.chkey + cs * B.HC;
  const uint32_t* G = B.chgen + cs * B.HC;
  const uint32_t* I = B.chidx + cs * B.HC;
  uint32_t h = hmix(key) & (uint32_t)(B.HC - 1);
  for (int probe = 0; probe < B.HC; ++probe) {
    const uint32_t g = G[h], ix = I[h];   // the slot's three words in one round trip
    const uint64_t k = K[h];
    if (g != gen) return -1;
    if (k == key) return (int)ix;
    h = (h + 1) & (uint32_t)(B.HC - 1);
  }
  return -1;
}
// insert a key known to be absent (keys inserted concurrently are distinct)
DEV void voxel_insert(const Batch& B, size_t cs, uint32_t gen, uint64_t key, uint32_t idx) {
  uint64_t* K = B.chkey + cs * B.HC;
  uint32_t* G = B.chgen + cs * B.HC;
  uint32_t* I = B.chidx + cs * B.HC;
  uint32_t h = hmix(key) & (uint32_t)(B.HC - 1);
  for (int probe = 0; probe < B.HC; ++probe) {
    const uint32_t g = G[h];
    if (g != gen && atomicCAS(&G[h], g, gen) == g) {
      K[h] = key;
      I[h] = idx;
      return;
    }
    if (g == gen || G[h] == gen) h = (h + 1) & (uint32_t)(B.HC - 1);
  }
}

DEV uint32_t pack_rgb(const uint8_t* rgb, int i) {
  return rgb ? ((uint32_t)rgb[3 * i] | (uint32_t)rgb[3 * i + 1] << 8 | (uint32_t)rgb[3 * i + 2] << 16) : (128u | 128u << 8 | 128u << 16);
}

DEV int vclampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// gatherRgbHost (bestview.cpp:84-92) of one point: the colour at its pixel, clamped to the
// image, packed r | g << 8 | b << 16 as the cloud stores it
DEV uint32_t gather_rgba(const uint8_t* rgba, const int32_t* px, int i, int w, int h) {
  const int x = vclampi(px[2 * i], 0, w - 1), y = vclampi(px[2 * i + 1], 0, h - 1);
  const uchar4 c = ((const uchar4*)rgba)[(size_t)y * w + x];
  return (uint32_t)c.x | (uint32_t)c.y << 8 | (uint32_t)c.z << 16;
}

// cap trim (cloud.cpp:114-123): std::nth_element(pts, pts + (n - keep), by seq), then the first
// n - keep elements are erased and the rest keep the order the selection left them in.  Later
// steps sample the cloud with a stride, so that order is an output: the selection reproduces
// libstdc++'s (the reference's build): median-of-three pivot moved to the front, unguarded
// Hoare partition, depth limit 2 floor(log2 n), insertion sort below four elements.  Each
// partition is computed in parallel from its two stopping sequences: with L = positions whose
// key is >= the pivot (ascending) and R = positions whose key is <= the pivot (descending), the
// sequential loop swaps L[i] <-> R[i] while L[i] < R[i], and returns L[0] when it made no swap,
// else min(L[k], R[k-1]) after k swaps.  (tests/trim_order_check.cpp checks the rule against
// std::nth_element.)  Elements are (seq << 32 | index) words; only seq is compared.
DEV bool trim_lt(uint64_t a, uint64_t b) { return (uint32_t)(a >> 32) < (uint32_t)(b >> 32); }

DEV void cloud_trim(const Batch& B, size_t cs, const Work& W, int* hist, BlockScratch& bs) {
  CloudRec& C = B.clouds[cs];
  const int cap = B.p.cloud_cap;
  const int n = C.n;
  if (cap <= 0 || n <= cap) return;
  const int keep = max(1, cap * 9 / 10), nth = n - keep;
  float4* pts = B.cpts + cs * B.cap;
  uint32_t* col = B.crgb + cs * B.cap;
  uint64_t* E = W.keys;               // the elements being selected
  int32_t* PL = W.dst;                // L positions, ascending
  int32_t* PR = (int32_t*)W.tab;      // R positions, ascending (R[i] = PR[nR - 1 - i])
  for (int i = threadIdx.x; i < n; i += blockDim.x) E[i] = ((uint64_t)__float_as_uint(pts[i].w) << 32) | (uint32_t)i;
  __shared__ int s_first, s_last, s_depth, s_fail;
  __shared__ int trim_db[2][33];
  int trim_it = 0;
  if (threadIdx.x == 0) {
    s_first = 0;
    s_last = n;
    int lg = 0;
    for (int v = n; v > 1; v >>= 1) ++lg;
    s_depth = 2 * lg;
    s_fail = 0;
  }
  __syncthreads();
  while (true) {
    const int first = s_first, last = s_last;
    if (last - first <= 3) break;
    if (threadIdx.x == 0) {
      if (s_depth == 0) {
        s_fail = 1;
      } else {
        --s_depth;
        const int x = first + 1, y = first + (last - first) / 2, z = last - 1;
        int md;
        if (trim_lt(E[x], E[y])) md = trim_lt(E[y], E[z]) ? y : (trim_lt(E[x], E[z]) ? z : x);
        else md = trim_lt(E[x], E[z]) ? x : (trim_lt(E[y], E[z]) ? z : y);
        const uint64_t t = E[first]; E[first] = E[md]; E[md] = t;
      }
    }
    __syncthreads();
    if (s_fail) break;
    const uint64_t pv = E[first];
    int nL = 0, nR = 0;
    for (int c0 = first + 1; c0 < last; c0 += blockDim.x) {
      const int j = c0 + threadIdx.x;
      const bool in = j < last;
      const uint64_t e = in ? E[j] : 0;
      const int fl = in && !trim_lt(e, pv), fr = in && !trim_lt(pv, e);
      int tl, tr;
      const int ol = block_scan_db(fl, &tl, trim_db, trim_it++);
      const int orr = block_scan_db(fr, &tr, trim_db, trim_it++);
      if (fl && INB(nL + ol, B.work_n, 421)) PL[nL + ol] = j;
      if (fr && INB(nR + orr, B.work_n, 422)) PR[nR + orr] = j;
      nL += tl;
      nR += tr;
    }
    __syncthreads();
    // swaps made: the pairs i with L[i] < R[i] (a prefix of the pairs)
    const int np = min(nL, nR);
    int cnt = 0;
    for (int i = threadIdx.x; i < np; i += blockDim.x) cnt += PL[i] < PR[nR - 1 - i];
    const int k = block_sum_i(cnt, bs);
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
      const int l = PL[i], r = PR[nR - 1 - i];
      const uint64_t t = E[l]; E[l] = E[r]; E[r] = t;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      const int cut = k == 0 ? PL[0] : min(k < nL ? PL[k] : last, PR[nR - k]);
      if (cut <= nth) s_first = cut;
      else s_last = cut;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    if (s_fail) {
      // the depth limit ran out (the reference would switch to a heap selection): keep the
      // newest points in storage order and report it
      set_err(&B.maps[cs / B.O], SMG_E_TRIM);
    } else {
      for (int i = s_first + 1; i < s_last; ++i) {   // stable insertion sort of the last few
        const uint64_t v = E[i];
        int j = i;
        while (j > s_first && trim_lt(v, E[j - 1])) { E[j] = E[j - 1]; --j; }
        E[j] = v;
      }
    }
  }
  __syncthreads();
  int w = 0;
  if (!s_fail) {
    for (int i = threadIdx.x; i < keep; i += blockDim.x) {
      const int src = (int)(uint32_t)E[nth + i];
      if (INB(src, n, 404)) { W.t4[i] = pts[src]; W.tc[i] = col[src]; }
    }
    w = keep;
  } else {   // fallback: the keep newest in storage order
    for (int i = threadIdx.x; i < n; i += blockDim.x) W.scr[i] = (double)__float_as_uint(pts[i].w);
    __syncthreads();
    const double cut = block_select(W.scr, n, nth, hist, bs);
    int lt = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) lt += W.scr[i] < cut;
    const int eq_drop = nth - block_sum_i(lt, bs);
    int eq_seen = 0;
    for (int c0 = 0; c0 < n; c0 += blockDim.x) {
      const int i = c0 + threadIdx.x;
      const int is_eq = i < n && W.scr[i] == cut;
      int toteq;
      const int peq = block_scan_db(is_eq, &toteq, trim_db, trim_it++);
      const int k = i < n && (W.scr[i] > cut || (is_eq && eq_seen + peq >= eq_drop));
      int tot;
      const int pos = block_scan_db(k, &tot, trim_db, trim_it++);
      if (k && INB(w + pos, B.work_n, 404)) { W.t4[w + pos] = pts[i]; W.tc[w + pos] = col[i]; }
      w += tot;
      eq_seen += toteq;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < w; i += blockDim.x) { pts[i] = W.t4[i]; col[i] = W.tc[i]; }
  __shared__ uint32_t sh_gen;
  if (threadIdx.x == 0) { C.n = w; sh_gen = ++C.vgen; }
  __syncthreads();
  for (int i = threadIdx.x; i < w; i += blockDim.x)
    voxel_insert(B, cs, sh_gen, voxel_key(pts[i].x, pts[i].y, pts[i].z, B.inv_vox_cloud), (uint32_t)i);
  __syncthreads();
}

// ObjCloud::add of n map-frame points (float xyz; colours from rgb, 3 bytes a point, or gathered
// from an RGBA image at the points' pixels px, or grey).  Block-wide.
DEV void cloud_add(const Batch& B, int m, size_t cs, const float* xyz, const uint8_t* rgb, int n, double stamp, const Work& W,
                   int* hist, BlockScratch& bs, const int32_t* px = nullptr, const uint8_t* rgba = nullptr, int iw = 0,
                   int ih = 0) {
  if (n <= 0) return;
  CloudRec& C = B.clouds[cs];
  const int tid = threadIdx.x;
  if (n > B.work_n) {
    if (tid == 0) set_err(&B.maps[m], SMG_E_CAP_PTS);
    return;
  }
  __shared__ uint32_t sh_seq, sh_vgen;
  __shared__ double sh_org[3];
  __shared__ int sh_base;
  if (tid == 0) {
    if (!C.has_org) {
      for (int k = 0; k < 3; ++k) C.org[k] = (double)xyz[k];
      C.has_org = 1;
    }
    sh_seq = ++C.seq;
    sh_vgen = C.vgen;
    sh_base = C.n;
    for (int k = 0; k < 3; ++k) sh_org[k] = C.org[k];
  }
  int hs = 1;
  while (hs < 2 * n) hs <<= 1;
  for (int i = tid; i < hs; i += blockDim.x) { W.tab[i].key = ~0ull; W.tab[i].first = 0xffffffffu; W.tab[i].last = 0; }
  __syncthreads();
  const float inv = B.inv_vox_cloud;
  for (int i = tid; i < n; i += blockDim.x) {
    const float x = (float)((double)xyz[3 * i] - sh_org[0]), y = (float)((double)xyz[3 * i + 1] - sh_org[1]),
                z = (float)((double)xyz[3 * i + 2] - sh_org[2]);
    const uint64_t key = voxel_key(x, y, z, inv);
    W.keys[i] = key;
    uint32_t h = hmix(key) & (uint32_t)(hs - 1);
    for (int probe = 0; probe < hs; ++probe) {
      const unsigned long long prev = atomicCAS(&W.tab[h].key, ~0ull, (unsigned long long)key);
      if (prev == ~0ull || prev == key) {
        atomicMin(&W.tab[h].first, (uint32_t)i);
        atomicMax(&W.tab[h].last, (uint32_t)i);
        break;
      }
      h = (h + 1) & (uint32_t)(hs - 1);
    }
  }
  __syncthreads();
  const int base = sh_base;
  float4* pts = B.cpts + cs * B.cap;
  uint32_t* col = B.crgb + cs * B.cap;
  int added = 0;
  __shared__ int sh_nw;
  __shared__ int add_db[2][33];
  int add_it = 0;
  if (tid == 0) sh_nw = 0;
  __syncthreads();
  for (int c0 = 0; c0 < n; c0 += blockDim.x) {
    const int i = c0 + tid;
    int isnew = 0, last = -1, old = -1;
    if (i < n) {
      const uint64_t key = W.keys[i];
      uint32_t h = hmix(key) & (uint32_t)(hs - 1);
      for (int probe = 0; probe < hs && W.tab[h].key != key; ++probe) h = (h + 1) & (uint32_t)(hs - 1);
      if (W.tab[h].first == (uint32_t)i) {
        last = (int)W.tab[h].last;
        old = voxel_lookup(B, cs, sh_vgen, key);
        isnew = old < 0;
      }
    }
    int tot;
    const int pos = block_scan_db(isnew, &tot, add_db, add_it++);
    if (i < n) W.dst[i] = -1;
    if (last >= 0) {
      const int d = isnew ? base + added + pos : old;
      if (d < B.cap && INB(d, B.cap, 401) && INB(last, n, 402)) {
        const float x = (float)((double)xyz[3 * last] - sh_org[0]), y = (float)((double)xyz[3 * last + 1] - sh_org[1]),
                    z = (float)((double)xyz[3 * last + 2] - sh_org[2]);
        pts[d] = make_float4(x, y, z, __uint_as_float(sh_seq));
        col[d] = rgba && !rgb ? gather_rgba(rgba, px, last, iw, ih) : pack_rgb(rgb, last);
        atomicAdd(&sh_nw, 1);
        if (isnew) W.dst[i] = d;
      }
    }
    added += tot;
  }
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x)
    if (W.dst[i] >= 0 && INB(W.dst[i], B.cap, 403)) voxel_insert(B, cs, sh_vgen, W.keys[i], (uint32_t)W.dst[i]);
  __syncthreads();
  if (tid == 0) {
    wk_add(&B.maps[m], SMG_WK_CLOUD, sh_nw);
    C.n = base + added;
    if (C.n > B.cap) { C.n = B.cap; set_err(&B.maps[m], SMG_E_CAP_PTS); }
  }
  __syncthreads();
  cloud_trim(B, cs, W, hist, bs);
  if (tid == 0) {
    ++C.version;
    C.stamp = stamp;
  }
  __syncthreads();
}

// apBuildContact over the cloud's map-frame points float(org + p) (objmap.cpp:1090-1103).
// Two representations of the same cell set: a dilated occupancy bitset over the cell box
// [lo-1, hi+1] (bit = some cloud cell within the 27-neighbourhood, so a contact test is one bit)
// when the box fits CB_WORDS words, else a generation-tagged hash set (racing duplicates of one
// key only cost a slot).
DEV void contact_rebuild(const Batch& B, size_t cs, BlockScratch& bs) {
  CloudRec& C = B.clouds[cs];
  const int n = C.n;
  const double inv = 1.0 / B.p.contact_cell;
  const float4* pts = B.cpts + cs * B.cap;
  auto cell = [&](int i, long long c[3]) {
    const float4 p = pts[i];
    const float q[3] = {(float)(C.org[0] + (double)p.x), (float)(C.org[1] + (double)p.y), (float)(C.org[2] + (double)p.z)};
    for (int k = 0; k < 3; ++k) c[k] = (long long)floor((double)q[k] * inv);
  };
  double lo[3] = {1e300, 1e300, 1e300}, hi[3] = {-1e300, -1e300, -1e300};
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    long long c[3];
    cell(i, c);
    for (int k = 0; k < 3; ++k) { lo[k] = fmin(lo[k], (double)c[k]); hi[k] = fmax(hi[k], (double)c[k]); }
  }
  long long L[3], H[3];
  for (int k = 0; k < 3; ++k) {
    L[k] = (long long)block_min_d(lo[k], bs);
    H[k] = (long long)block_max_d(hi[k], bs);
  }
  const long long dx = H[0] - L[0] + 3, dy = H[1] - L[1] + 3, dz = H[2] - L[2] + 3;
  const long long wpr = (dx + 31) / 32;
  const bool fits = n > 0 && wpr * dy * dz <= CB_WORDS;
  __shared__ uint32_t sh_gen;
  if (threadIdx.x == 0) {
    for (int k = 0; k < 3; ++k) { C.clo[k] = n > 0 ? L[k] : 0; C.chi[k] = n > 0 ? H[k] : -1; }
    C.cb_ok = fits;
    C.cb_dy = (int)dy;
    C.cb_dz = (int)dz;
    C.cb_wpr = (int)wpr;
    sh_gen = fits ? C.cgen : ++C.cgen;
  }
  __syncthreads();
  if (fits) {
    uint32_t* O = B.cbits + cs * 2 * CB_WORDS;
    uint32_t* D = O + CB_WORDS;
    const int words = (int)(wpr * dy * dz);
    for (int i = threadIdx.x; i < words; i += blockDim.x) { O[i] = 0; D[i] = 0; }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      long long c[3];
      cell(i, c);
      const int x = (int)(c[0] - L[0] + 1), y = (int)(c[1] - L[1] + 1), z = (int)(c[2] - L[2] + 1);
      const size_t w = ((size_t)z * dy + y) * wpr + (x >> 5);
      if (INB(w, (size_t)words, 420)) atomicOr(&O[w], 1u << (x & 31));
    }
    __syncthreads();
    // dilate along x (with carries across words), then y, then z
    for (int i = threadIdx.x; i < words; i += blockDim.x) {
      const int wx = (int)(i % wpr);
      const uint32_t w = O[i];
      const uint32_t prev = wx > 0 ? O[i - 1] : 0u, next = wx + 1 < wpr ? O[i + 1] : 0u;
      D[i] = w | (w << 1) | (w >> 1) | (prev >> 31) | (next << 31);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < words; i += blockDim.x) {
      const long long row = i / wpr, y = row % dy;
      const uint32_t up = y > 0 ? D[i - wpr] : 0u, dn = y + 1 < dy ? D[i + wpr] : 0u;
      O[i] = D[i] | up | dn;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < words; i += blockDim.x) {
      const long long z = i / (wpr * dy);
      const uint32_t below = z > 0 ? O[i - wpr * dy] : 0u, above = z + 1 < dz ? O[i + wpr * dy] : 0u;
      D[i] = O[i] | below | above;
    }
  } else {
    const uint32_t gen = sh_gen;
    uint64_t* K = B.ckey + cs * B.HCC;
    uint32_t* G = B.cgen + cs * B.HCC;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      long long c[3];
      cell(i, c);
      const uint64_t key = cell_key3(c[0], c[1], c[2]);
      uint32_t h = hmix(key) & (uint32_t)(B.HCC - 1);
      for (int probe = 0; probe < B.HCC; ++probe) {
        const uint32_t g = G[h];
        if (g == gen) {
          if (K[h] == key) break;
        } else if (atomicCAS(&G[h], g, gen) == g) {
          K[h] = key;
          break;
        } else {
          continue;   // lost the slot to another writer: look at it again
        }
        h = (h + 1) & (uint32_t)(B.HCC - 1);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) { C.cn = n; C.cver = C.version; }
  __syncthreads();
}

// Cloud additions of the frame: CTA j of map m adds, in emission order, every observation
// cloud of target object j (ObjectMap::addPoints, objmap.cpp:508-514 via capi.cpp:986-992), then
// rebuilds its contact index.  Targets also include objects whose cloud moved (translate).
__global__ void __launch_bounds__(512) k_cloud_add(Batch B) {
  __shared__ BlockScratch bs;
  __shared__ int hist[SEL_HIST(1)];
  const int m = B.map0 + blockIdx.y;
  const FrameDev& F = B.frames[m];
  if (!F.active) return;
  const MapRec& R = B.maps[m];
  const Work W = work_at(B, m, blockIdx.x);
  PHASE_START();
  for (int j = blockIdx.x; j < R.n_targets; j += gridDim.x) {
    if (!INB(j, B.O, 405)) break;
    const int slot = B.tgt_slot[(size_t)m * B.O + j];
    if (!INB(slot, B.O, 406)) continue;
    const ObjRec& o = B.objs[oglob(B, m, slot)];
    const size_t cs = cglob(B, m, o.cloud_slot);
    for (int e = 0; e < R.n_pts; ++e) {
      if (!INB(e, B.max_det, 407)) break;
      const PtsRec& pr = B.ptsl[(size_t)m * B.max_det + e];
      if (pr.obj_id != o.id) continue;
      if (!INB(pr.det, B.max_det, 408) || !INB(pr.n, B.pmax + 1, 409)) continue;
      const float* xyz = B.cxyz + ((size_t)m * B.max_det + pr.det) * 3 * B.pmax;
      const int32_t* px = B.cpx + ((size_t)m * B.max_det + pr.det) * 2 * B.pmax;
      cloud_add(B, m, cs, xyz, nullptr, pr.n, F.stamp, W, hist, bs, px, F.views_on ? F.rgba : nullptr, F.w, F.h);
    }
    PHASE_MARK(37);   // cloud additions of a target
    if (B.clouds[cs].cver != B.clouds[cs].version) contact_rebuild(B, cs, bs);
    PHASE_MARK(38);   // its contact index
  }
}
