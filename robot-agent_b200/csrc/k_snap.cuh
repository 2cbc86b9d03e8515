// Object-memory snapshot of every map in one pass (sm_snapshot's object list, scenemap
// capi.cpp:1051-1067, and dsg_save's per-object point files, dsg_save.cpp:70-89 plyBytes).
//
//  - k_snap_list: per map, the exportable objects (ObjectMap::exportable) in object order, by an
//    ordered block compaction; their sm_object fields and point counts.
//  - k_snap_scan: one CTA turns the per-map counts into map offsets and the objects' point
//    counts into record offsets (exclusive scans, 64-bit).
//  - k_snap_pack: the records to their packed places, and every exportable cloud's points as
//    15-byte PLY vertex records (float x, y, z in map metres, uchar r, g, b), a thread per point.
// The device packs, the host reads two contiguous buffers.
#pragma once
#include "dev_util.cuh"

#define SNAP_SCAN_THREADS 1024

__global__ void __launch_bounds__(256) k_snap_list(Batch B, smg_snap_object* rec, int32_t* cnt, int64_t* npts, int32_t* src) {
  __shared__ int scan_db[2][33];
  const int m = blockIdx.x;
  const MapRec& R = B.maps[m];
  const smg_params& P = B.p;
  const size_t base = (size_t)m * B.O;
  int before = 0, it = 0;
  for (int c0 = 0; c0 < R.n_obj; c0 += blockDim.x) {
    const int b = c0 + threadIdx.x;
    const ObjRec* o = nullptr;
    int need = 0;
    if (b < R.n_obj) {
      o = &B.objs[oglob(B, m, slot_at(B, m, b))];
      need = exportable(B, *o);
    }
    int tot;
    const int r = before + block_scan_db(need, &tot, scan_db, it++);
    if (need && INB(r, B.O, 1201)) {
      smg_snap_object e;
      e.id = o->id;
      e.name_lab = o->cls >= 0 && o->cls < B.txt.n_labels ? o->cls : -1;
      e.score = o->score;
      for (int k = 0; k < 3; ++k) { e.pos[k] = o->pos[k]; e.extent[k] = o->ext[k]; e.first_pos[k] = o->first_pos[k]; }
      e.n_obs = o->n_obs;
      e.last_seen = o->last_seen;
      e.state = o->held_by >= 0 ? 3 : o->state;   // SM_HELD
      const int kd = kind_of(B, o->cls);
      e.structural = kd == KIND_STATIC || kd == KIND_STRUCT_OBJ || smax3(o->ext[0], o->ext[1], o->ext[2]) > P.big;
      e.movable = kd != KIND_STATIC && kd != KIND_STRUCT_OBJ;
      const CloudRec& C = B.clouds[cglob(B, m, o->cloud_slot)];
      e.n_points = C.n;
      e.cloud_stamp = C.stamp;
      rec[base + r] = e;
      npts[base + r] = C.n;
      src[base + r] = o->cloud_slot;
    }
    before += tot;
  }
  if (threadIdx.x == 0) cnt[m] = min(before, B.O);
}

// map_off[m] = objects of maps < m (M + 1 entries); pt_off[i] = points of packed objects < i
// (n_total + 1 entries), the packed order being map after map
__global__ void __launch_bounds__(SNAP_SCAN_THREADS) k_snap_scan(Batch B, const int32_t* cnt, const int64_t* npts, int32_t* map_off,
                                                                 int64_t* pt_off) {
  __shared__ long long part[SNAP_SCAN_THREADS / 32];
  __shared__ long long s_carry;
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int m = 0; m < B.M; ++m) { map_off[m] = acc; acc += cnt[m]; }
    map_off[B.M] = acc;
    s_carry = 0;
  }
  __syncthreads();
  const int n = map_off[B.M];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int c0 = 0; c0 < n; c0 += blockDim.x) {
    const int i = c0 + threadIdx.x;
    long long v = 0;
    if (i < n) {   // packed object i: map m with map_off[m] <= i < map_off[m + 1]
      int lo = 0, hi = B.M - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (map_off[mid] <= i) lo = mid; else hi = mid - 1;
      }
      v = npts[(size_t)lo * B.O + (i - map_off[lo])];
    }
    long long x = v;
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) part[wid] = x;
    __syncthreads();
    long long before = s_carry;
    for (int w = 0; w < wid; ++w) before += part[w];
    if (i < n) pt_off[i] = before + x - v;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) s_carry = before + x;
    __syncthreads();
  }
  if (threadIdx.x == 0) pt_off[n] = s_carry;
}

// grid (objects chunk, map): records to their packed places, points to 15-byte vertex records
__global__ void __launch_bounds__(256) k_snap_pack(Batch B, const smg_snap_object* rec, const int32_t* cnt, const int32_t* src,
                                                   const int32_t* map_off, const int64_t* pt_off, smg_snap_object* out_rec,
                                                   uint8_t* out_pts) {
  const int m = blockIdx.y;
  const int n = cnt[m];
  const size_t base = (size_t)m * B.O;
  for (int r = blockIdx.x; r < n; r += gridDim.x) {
    const int g = map_off[m] + r;
    if (threadIdx.x == 0 && out_rec) out_rec[g] = rec[base + r];
    if (!out_pts) continue;
    const size_t cs = cglob(B, m, src[base + r]);
    const CloudRec& C = B.clouds[cs];
    const float4* pts = B.cpts + cs * B.cap;
    const uint32_t* col = B.crgb + cs * B.cap;
    uint8_t* dst = out_pts + (size_t)pt_off[g] * 15;
    for (int i = threadIdx.x; i < C.n; i += blockDim.x) {
      const float4 q = pts[i];
      const float xyz[3] = {(float)(C.org[0] + (double)q.x), (float)(C.org[1] + (double)q.y), (float)(C.org[2] + (double)q.z)};
      const uint32_t c = col[i];
      uint8_t* p = dst + (size_t)i * 15;
      for (int k = 0; k < 3; ++k) {
        const uint32_t u = __float_as_uint(xyz[k]);
        p[4 * k] = (uint8_t)u;
        p[4 * k + 1] = (uint8_t)(u >> 8);
        p[4 * k + 2] = (uint8_t)(u >> 16);
        p[4 * k + 3] = (uint8_t)(u >> 24);
      }
      p[12] = (uint8_t)(c & 255u);
      p[13] = (uint8_t)((c >> 8) & 255u);
      p[14] = (uint8_t)((c >> 16) & 255u);
    }
  }
}
