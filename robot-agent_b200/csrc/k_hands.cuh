// ObjectMap::updateHands (scenemap src/objmap.cpp:435-506), the first step of ObjectMap::update
// (:517): grasp, hold and release by the robot's gripper(s), and objects that rest on / in another
// object following it.
//
// The per-hand gripper state machine (closed, settled, tried once per closure) depends only on
// the gripper values and stamps, so the host runs it and FrameDev carries, per hand, what this
// frame does: try a grasp (bit 0), release because the gripper closed to the end after a grasp
// (bit 1), release because it opened (bit 2), and the finger gap of gripGap.
//
// One CTA per map.  The grasp search (nearest holdable object within grasp_r, first in list
// order on ties) and the held objects' motion run over all threads; releases and the support
// links run on thread 0 in list order, as the reference's loops do (a support found by a later
// object can itself have moved earlier in the same loop).
#pragma once
#include "k_cloud.cuh"

#define HANDS_THREADS 128

// ObjCloud::translate (cloud.cpp:79-84) along axis k only, as the reference calls it once per axis
DEV void cloud_translate_axis(const Batch& B, int m, const ObjRec& o, int k, double dk, double t) {
  CloudRec& C = B.clouds[cglob(B, m, o.cloud_slot)];
  if (C.n <= 0 || dk == 0) return;
  C.org[k] += dk;
  ++C.version;
  C.stamp = t;
}

// holdable (objmap.cpp:400-410): not big, middle side <= grasp_max_w, the gap fits the sides
DEV bool holdable(const Batch& B, const ObjRec& o, double gap) {
  const smg_params& P = B.p;
  if (is_big(B, o)) return false;
  double e[3];
  for (int k = 0; k < 3; ++k) e[k] = smax(0.0, o.hi[k] - o.lo[k]);
  // sort the three sides
  if (e[0] > e[1]) { const double x = e[0]; e[0] = e[1]; e[1] = x; }
  if (e[1] > e[2]) { const double x = e[1]; e[1] = e[2]; e[2] = x; }
  if (e[0] > e[1]) { const double x = e[0]; e[0] = e[1]; e[1] = x; }
  if (e[1] > P.grasp_max_w) return false;
  if (gap < P.grasp_min_gap) return false;
  return gap >= e[0] - P.grasp_w_tol && gap <= e[2] + P.grasp_w_tol;
}

// release (objmap.cpp:412-433): thread 0 only
DEV void hand_release(const Batch& B, int m, int pos, double t, int* evn) {
  const smg_params& P = B.p;
  const MapRec& R = B.maps[m];
  ObjRec& o = B.objs[oglob(B, m, slot_at(B, m, pos))];
  o.held_by = -1;
  const bool mv = dist3(o.pos, o.grasp_pos) > P.moved_d;
  o.moved = o.moved || mv;
  o.state = o.moved ? 2 : 0;
  o.misses = 0;
  int best = -1;
  double bv = 1e18;
  for (int i = 0; i < R.n_obj; ++i) {
    if (i == pos) continue;
    const ObjRec& p = obj_at(B, m, i);
    if (!p.confirmed || p.state == 1) continue;
    if (o.pos[0] < p.lo[0] - 0.1 || o.pos[0] > p.hi[0] + 0.1 || o.pos[1] < p.lo[1] - 0.1 || o.pos[1] > p.hi[1] + 0.1) continue;
    if (o.pos[2] < p.lo[2] - 0.05) continue;
    const double v = o.pos[2] - smin(p.hi[2], o.pos[2]);
    if (v < bv) { bv = v; best = i; }
  }
  if (best >= 0) {
    const ObjRec& p = obj_at(B, m, best);
    o.parent = p.id;
    for (int k = 0; k < 3; ++k) o.parent_rel[k] = o.pos[k] - p.pos[k];
  }
  push_event(B, m, t, o, 5, (0u << 24) | (uint32_t)(*evn)++);
}

__global__ void __launch_bounds__(HANDS_THREADS) k_hands(Batch B) {
  __shared__ double s_bd[HANDS_THREADS];
  __shared__ int s_bi[HANDS_THREADS];
  __shared__ int s_any;
  __shared__ BlockScratch bs;
  const int m = B.map0 + blockIdx.x, tid = threadIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active || !F.hands_on) return;
  const smg_params& P = B.p;
  const MapRec& R = B.maps[m];
  const int n = R.n_obj;
  const double t = F.stamp, cy = F.cos_th, sy = F.sin_th;
  int evn = 0;   // thread 0's event counter (phase 0: before the merge pass)
  for (int h = 0; h < 2; ++h) {
    const int act = F.hand_act[h];
    if (act & 1) {   // grasp: the nearest holdable confirmed object within grasp_r (objmap.cpp:455-465)
      double bd = P.grasp_r;
      int bi = -1;
      for (int i = tid; i < n; i += blockDim.x) {
        const ObjRec& o = obj_at(B, m, i);
        if (!o.confirmed || o.held_by >= 0 || o.state == 1) continue;
        const double d = dist3(o.pos, F.eef[h]);
        if (d < bd && holdable(B, o, F.hand_gap[h])) { bd = d; bi = i; }   // a thread's i ascend: first on ties
      }
      s_bd[tid] = bd;
      s_bi[tid] = bi;
      __syncthreads();
      if (tid == 0) {
        for (int q = 1; q < blockDim.x; ++q)
          if (s_bi[q] >= 0 && (s_bi[0] < 0 || s_bd[q] < s_bd[0] || (s_bd[q] == s_bd[0] && s_bi[q] < s_bi[0]))) {
            s_bd[0] = s_bd[q];
            s_bi[0] = s_bi[q];
          }
        if (s_bi[0] >= 0) {   // grab (objmap.cpp:437-447)
          ObjRec& o = B.objs[oglob(B, m, slot_at(B, m, s_bi[0]))];
          o.held_by = h;
          o.parent = 0;
          const double d[3] = {o.pos[0] - F.eef[h][0], o.pos[1] - F.eef[h][1], o.pos[2] - F.eef[h][2]};
          o.held_rel[0] = cy * d[0] + sy * d[1];
          o.held_rel[1] = -sy * d[0] + cy * d[1];
          o.held_rel[2] = d[2];
          for (int k = 0; k < 3; ++k) o.grasp_pos[k] = o.pos[k];
          o.state = 3;
          push_event(B, m, t, o, 4, (0u << 24) | (uint32_t)evn++);
        }
      }
      __syncthreads();
    }
    if ((act & 6) && tid == 0)   // releases in list order: closed to the end (bit 1), opened (bit 2)
      for (int pass = 1; pass <= 2; ++pass) {
        if (!(act & (2 << (pass - 1)))) continue;
        for (int i = 0; i < n; ++i)
          if (obj_at(B, m, i).held_by == h) hand_release(B, m, i, t, &evn);
      }
    __syncthreads();
  }
  // held objects follow the hand, rotated with the base (objmap.cpp:474-486)
  if (tid == 0) s_any = 0;
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) {
    ObjRec& o = B.objs[oglob(B, m, slot_at(B, m, i))];
    if (o.parent) s_any = 1;
    if (o.held_by < 0) continue;
    const double* r = o.held_rel;
    for (int k = 0; k < 3; ++k) {
      const double rel = k == 0 ? cy * r[0] - sy * r[1] : (k == 1 ? sy * r[0] + cy * r[1] : r[2]);
      const double np = F.eef[o.held_by][k] + rel, dk = np - o.pos[k];
      o.pos[k] = np;
      o.lo[k] += dk;
      o.hi[k] += dk;
      cloud_translate_axis(B, m, o, k, dk, t);
    }
  }
  __syncthreads();
  // objects put on / in another one follow it (objmap.cpp:488-505), list order
  if (tid == 0 && s_any)
    for (int i = 0; i < n; ++i) {
      ObjRec& o = B.objs[oglob(B, m, slot_at(B, m, i))];
      if (!o.parent) continue;
      int pi = -1;
      for (int q = 0; q < n; ++q)
        if (obj_at(B, m, q).id == o.parent) { pi = q; break; }
      if (pi < 0) { o.parent = 0; continue; }
      const ObjRec& p = obj_at(B, m, pi);
      for (int k = 0; k < 3; ++k) {
        const double np = p.pos[k] + o.parent_rel[k], dk = np - o.pos[k];
        if (fabs(dk) > 1e-9) o.moved = 1;
        o.pos[k] = np;
        o.lo[k] += dk;
        o.hi[k] += dk;
        cloud_translate_axis(B, m, o, k, dk, t);
      }
      if (o.moved && o.state == 0) o.state = 2;
    }
  __syncthreads();
  // A moved cloud's contact cells move with it: the reference rebuilds its contact index on
  // demand from the new cloud version (objmap.cpp:1090-1103); the merge pass and association of
  // this frame read it, so it is rebuilt here.  Every index is current at the start of a frame
  // (k_cloud_add rebuilds the stale ones), so a stale one now is a cloud moved above.
  for (int i = 0; i < n; ++i) {
    const size_t cs = cglob(B, m, obj_at(B, m, i).cloud_slot);
    if (B.clouds[cs].cver != B.clouds[cs].version) contact_rebuild(B, cs, bs);
    __syncthreads();
  }
}
