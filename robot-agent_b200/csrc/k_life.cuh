// Change detection and clean-up of one keyframe (scenemap src/objmap.cpp:1020-1084):
// absence evidence and misses (k_absent, one warp per object), relink of gone/appeared pairs
// (k_relink, per map), geometry of merged clouds (k_struct, apStructObject :1255-1350), drop and
// prune plus the cloud-addition target list (k_prune, per map), and the seen-cells record
// (k_markview, markView :219-245).
#pragma once
#include "k_cloud.cuh"
#include "k_obs.cuh"

// toCam of absentEvidence (objmap.cpp:256-261)
DEV void to_cam(const double* T, const double p[3], double c[3]) {
  const double d[3] = {p[0] - T[3], p[1] - T[7], p[2] - T[11]};
  c[0] = T[0] * d[0] + T[4] * d[1] + T[8] * d[2];
  c[1] = T[1] * d[0] + T[5] * d[1] + T[9] * d[2];
  c[2] = T[2] * d[0] + T[6] * d[1] + T[10] * d[2];
}

// absentEvidence (objmap.cpp:254-312), warp-level: 2 = not seen and the space behind is seen,
// 1 = should be seen but is not, 0 = cannot tell
DEV int absent_evidence_warp(const Batch& B, int m, const ObjRec& o, const FrameDev& F) {
  const smg_params& P = B.p;
  const double* T = F.T_mc;
  double cc[3];
  to_cam(T, o.pos, cc);
  if (cc[2] < 0.3 || cc[2] > (double)P.zmax) return 0;
  if (o.max_det_z > 0 && cc[2] > P.absent_det_k * o.max_det_z + 0.2) return 0;
  const size_t cs = cglob(B, m, o.cloud_slot);
  const CloudRec& C = B.clouds[cs];
  const int nc = C.n;
  const int K = max(8, P.absent_samples);
  int ns;
  size_t stride = 1;
  if (nc >= 8) {
    stride = (size_t)nc / (size_t)K > 1 ? (size_t)nc / (size_t)K : 1;
    ns = (int)(((size_t)nc + stride - 1) / stride);
    if (ns > K) ns = K;
  } else {
    ns = 27;
  }
  const int lane = threadIdx.x & 31;
  int vis = 0, thru = 0;
  double u0 = 1e9, v0 = 1e9, u1 = -1e9, v1 = -1e9;
  const float4* pts = B.cpts + cs * B.cap;
  for (int s = lane; s < ns; s += 32) {
    double p[3];
    if (nc >= 8) {
      if (!INB((size_t)s * stride, nc, 504)) continue;
    const float4 q = pts[(size_t)s * stride];
      p[0] = C.org[0] + (double)q.x; p[1] = C.org[1] + (double)q.y; p[2] = C.org[2] + (double)q.z;
    } else {
      const int a = s / 9, b = (s / 3) % 3, c = s % 3;
      p[0] = o.lo[0] + 0.5 * a * (o.hi[0] - o.lo[0]);
      p[1] = o.lo[1] + 0.5 * b * (o.hi[1] - o.lo[1]);
      p[2] = o.lo[2] + 0.5 * c * (o.hi[2] - o.lo[2]);
    }
    double c[3];
    to_cam(T, p, c);
    if (c[2] < 0.2) continue;
    const double uf = (double)F.fx * c[0] / c[2] + (double)F.cx, vf = (double)F.fy * c[1] / c[2] + (double)F.cy;
    const int u = (int)uf, v = (int)vf;
    if (u < 2 || v < 2 || u >= F.w - 2 || v >= F.h - 2) continue;
    const float d = (F.depth_host ? F.depth_host : F.depth)[(size_t)v * F.w + u];   // host frame when gathered
    if (!(d > 0)) continue;
    if ((double)d < c[2] - P.occl) continue;
    ++vis;
    if ((double)d > c[2] + smax(P.occl, 0.1)) ++thru;
    u0 = smin(u0, uf); u1 = smax(u1, uf); v0 = smin(v0, vf); v1 = smax(v1, vf);
  }
  vis = warp_sum_i(vis);
  thru = warp_sum_i(thru);
  u0 = warp_min_d(u0); v0 = warp_min_d(v0); u1 = warp_max_d(u1); v1 = warp_max_d(v1);
  if (vis < max(3, (int)(P.absent_vis * ns + 0.5))) return 0;
  if (sqrt(smax(0.0, u1 - u0) * smax(0.0, v1 - v0)) < P.absent_min_px) return 0;
  return thru * 10 >= vis * 3 ? 2 : 1;
}


// absence and misses (objmap.cpp:1021-1061), one warp per object in list order
__global__ void __launch_bounds__(256) k_absent(Batch B) {
  const int m = B.map0 + blockIdx.y;
  const FrameDev& F = B.frames[m];
  if (!F.active) return;
  MapRec* R = &B.maps[m];
  const smg_params& P = B.p;
  const double* T = F.T_mc;
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), nwarps = gridDim.x * (blockDim.x >> 5);
  for (int b = gw; b < R->n_obj; b += nwarps) {
    ObjRec& o = B.objs[oglob(B, m, slot_at(B, m, b))];
    if (!o.confirmed || o.held_by >= 0 || B.obj_hit[(size_t)m * B.O + b] || o.state == 1) continue;
    if (o.parent) continue;   // an object put on / in another one stays where it was put
    if (dist3(o.pos, F.eef[0]) < (double)P.hand_r + 0.1 || dist3(o.pos, F.eef[1]) < (double)P.hand_r + 0.1) continue;
    const int ev = absent_evidence_warp(B, m, o, F);
    if (lane != 0 || !ev || B.touched[(size_t)m * B.O + b]) continue;
    const double cam_now[3] = {T[3], T[7], T[11]}, fwd[3] = {T[2], T[6], T[10]};
    if (o.misses > 0 && ev != 2) {
      const double cosang = fwd[0] * o.last_miss_fwd[0] + fwd[1] * o.last_miss_fwd[1] + fwd[2] * o.last_miss_fwd[2];
      if (dist3(cam_now, o.last_miss_cam) < P.gone_step_d && cosang > B.cos_gone_step) continue;
    }
    for (int k = 0; k < 3; ++k) { o.last_miss_cam[k] = cam_now[k]; o.last_miss_fwd[k] = fwd[k]; }
    const bool big = is_big(B, o);
    ++o.n_vis_miss;
    if (o.misses++ == 0) {
      o.first_miss = F.stamp;
      for (int k = 0; k < 3; ++k) o.miss_cam[k] = T[4 * k + 3];
    }
    const double pr = ((double)o.n_obs + 1.0) / ((double)o.n_obs + (double)o.n_vis_miss + 2.0);
    const int k_rate = pr >= 1.0 ? 0 : (int)ceil(log(P.gone_eps) / log(1.0 - pr));
    const int need = min(max(big ? P.gone_misses_big : P.gone_misses, k_rate), 60);
    const double need_s = big ? P.gone_min_s_big : P.gone_min_s;
    const bool indep = F.stamp - o.first_miss >= need_s - 1e-9 || dist3(cam_now, o.miss_cam) >= P.gone_view_d;
    if (o.misses >= need && indep) {
      o.state = 1;
      o.gone_t = F.stamp;
      o.n_vis_miss -= (uint32_t)min(o.misses, (int)o.n_vis_miss);
      push_event(B, m, F.stamp, o, 3, (3u << 24) | (uint32_t)b);
    }
  }
}

// remove list position `pos` (order kept); the object slot is freed, and the cloud slot too
// unless keep_cloud
DEV void erase_pos(const Batch& B, int m, int pos, bool keep_cloud) {
  MapRec* R = &B.maps[m];
  int32_t* ord = B.order + (size_t)m * B.O;
  const int slot = ord[pos];
  const ObjRec& o = B.objs[oglob(B, m, slot)];
  if (!INB(pos, R->n_obj, 501)) return;
  if (!keep_cloud) { if (INB(R->n_cfree, B.C, 502)) B.cfreel[(size_t)m * B.C + R->n_cfree++] = o.cloud_slot; }
  if (INB(R->n_free, B.O, 503)) B.freel[(size_t)m * B.O + R->n_free++] = slot;
  for (int i = pos + 1; i < R->n_obj; ++i) ord[i - 1] = ord[i];
  --R->n_obj;
}

DEV int find_pos(const Batch& B, int m, uint32_t id) {
  const MapRec& R = B.maps[m];
  for (int i = 0; i < R.n_obj; ++i)
    if (obj_at(B, m, i).id == id) return i;
  return -1;
}

// remapId (objmap.cpp:314-318) on this frame's association and cloud lists and on the objects'
// parent links
DEV void remap_id(const Batch& B, int m, uint32_t from, uint32_t to) {
  const MapRec& R = B.maps[m];
  const FrameDev& F = B.frames[m];
  for (int k = 0; k < F.n_det; ++k)
    if (B.assoc[(size_t)m * B.max_det + k].obj_id == from) B.assoc[(size_t)m * B.max_det + k].obj_id = to;
  for (int e = 0; e < R.n_pts; ++e)
    if (B.ptsl[(size_t)m * B.max_det + e].obj_id == from) B.ptsl[(size_t)m * B.max_det + e].obj_id = to;
  for (int i = 0; i < R.n_obj; ++i) {
    ObjRec& o = B.objs[oglob(B, m, slot_at(B, m, i))];
    if (o.parent == from) o.parent = to;
  }
}

#define RELINK_MAXC 256
#define STRUCT_CTAS 32
#define STRUCT_LIST 64
#define STRUCT_SCR (4096 + 2 * 4096)   // doubles per CTA: points (as floats) + plane-fit scratch
#define RELINK_STAGE 1024
// relink (objmap.cpp:321-385), per map: candidate pairs pass the scalar tests, a warp per pair
// evaluates the embedding cosine of n's mean direction against m, then pairs are applied nearest
// first.  Also emits the cloud-candidate list of the update (objmap.cpp:1010-1019) beforehand.
__global__ void __launch_bounds__(256) k_relink(Batch B) {
  __shared__ int cn_, cm_[RELINK_MAXC], cnn_[RELINK_MAXC];
  __shared__ double cd_[RELINK_MAXC], ccos_[RELINK_MAXC];
  __shared__ int np_;
  __shared__ double pd_[RELINK_MAXC];
  __shared__ uint32_t pm_[RELINK_MAXC], pn_[RELINK_MAXC];
  __shared__ int s_state[RELINK_STAGE], s_nobs[RELINK_STAGE], s_cls[RELINK_STAGE];
  __shared__ unsigned char s_flags[RELINK_STAGE];
  __shared__ double s_first[RELINK_STAGE], s_last[RELINK_STAGE];
  extern __shared__ unsigned char smem_raw[];
  double* s_pos = (double*)smem_raw;   // 3 per object
  const int m = B.map0 + blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
  const FrameDev& F = B.frames[m];
  if (!F.active) return;
  MapRec* R = &B.maps[m];
  const smg_params& P = B.p;
  const double t = F.stamp;
  if (wid == 0) {
    // cloud candidates in observation order (objmap.cpp:1010-1019): warp 0 loads 32
    // observations at a time and places the kept ones by a ballot prefix
    const int nobs = min(R->n_obs, B.max_det);
    int e = 0;
    for (int a0 = 0; a0 < nobs; a0 += 32) {
      const int a = a0 + lane;
      int det = 0, nc = 0;
      uint32_t id = 0;
      if (a < nobs) {
        det = B.obs_list[(size_t)m * B.max_det + a];
        if (INB(det, B.max_det, 513)) {
          id = B.assoc[(size_t)m * B.max_det + det].obj_id;
          nc = B.obs[(size_t)m * B.max_det + det].nc;
        }
      }
      const bool keep = a < nobs && id && nc > 0;
      const unsigned bal = __ballot_sync(0xffffffffu, keep);
      if (keep) {
        PtsRec& pr = B.ptsl[(size_t)m * B.max_det + e + __popc(bal & ((1u << lane) - 1u))];
        pr.obj_id = id;
        pr.det = det;
        pr.n = nc;
      }
      e += __popc(bal);
    }
    if (lane == 0) R->n_pts = e;
  }
  // stage the scalars of the relink tests (objmap.cpp:323-346) in shared memory
  const int nobj = R->n_obj;
  const bool staged = nobj <= RELINK_STAGE;
  for (int i = tid; i < nobj && staged; i += blockDim.x) {
    const ObjRec& o = obj_at(B, m, i);
    s_state[i] = o.state;
    s_flags[i] = (o.appeared ? 1 : 0) | (o.confirmed ? 2 : 0) | (o.moved ? 4 : 0) | (o.held_by >= 0 ? 8 : 0);
    s_nobs[i] = (int)o.n_obs;
    s_cls[i] = o.cls;
    s_first[i] = o.first_seen;
    s_last[i] = o.last_seen;
    for (int k = 0; k < 3; ++k) s_pos[3 * i + k] = o.pos[k];
  }
  __syncthreads();
  if (tid == 0) {
    if (!staged) set_err(R, SMG_E_CAP_OBJ);
    cn_ = 0;
  }
  __syncthreads();
  // scalar tests of the relink candidates (a pair needs a gone object m), one thread per n;
  // the candidates are sorted by (distance, m id, n id) below, so their list order is free
  for (int i = tid; staged && i < nobj; i += blockDim.x) {
    if (!(s_flags[i] & 1) || !(s_flags[i] & 2) || (s_flags[i] & 8) || s_state[i] == 1 || s_nobs[i] < P.link_min_obs) continue;
    if (t - s_first[i] > P.link_window_s) continue;
    for (int j = 0; j < nobj; ++j) {
      if (j == i || s_state[j] != 1 || !(s_flags[j] & 2) || (s_flags[j] & 8) || (!(s_flags[j] & 4) && s_nobs[j] < P.spurious_obs))
        continue;
      if (!(s_first[i] > s_last[j])) continue;
      const double d = dist3(&s_pos[3 * i], &s_pos[3 * j]);
      if (d > smin(P.link_max_d, P.link_d0 + P.link_v * (s_first[i] - s_last[j]))) continue;
      bool wait = false;
      if (t - s_first[i] < P.link_wait_s)
        for (int q = 0; q < nobj; ++q) {
          if (q == i || q == j || !(s_flags[q] & 2) || (s_flags[q] & 8) || s_state[q] == 1 || s_cls[q] != s_cls[i]) continue;
          if (s_last[q] < s_first[i] && dist3(&s_pos[3 * q], &s_pos[3 * i]) < d) { wait = true; break; }
        }
      if (wait) continue;
      const int c = atomicAdd(&cn_, 1);
      if (c < RELINK_MAXC) { cm_[c] = j; cnn_[c] = i; cd_[c] = d; }
      else set_err(R, SMG_E_ARGS);
    }
  }
  __syncthreads();
  if (tid == 0 && cn_ > RELINK_MAXC) cn_ = RELINK_MAXC;
  __syncthreads();
  // apCosMax(m, mu(n)) >= link_cos (mu = r_frag / |r_frag| as float, objprob.cpp:233-239): the
  // object's mu cache (kept current with r_frag by k_update_vec and the merge pass) is that vector
  for (int c = wid; c < cn_; c += nw) {
    const ObjRec& n = obj_at(B, m, cnn_[c]);
    const size_t ogn = oglob(B, m, slot_at(B, m, cnn_[c]));
    double cs = -3.0;
    if (n.nrm_frag > 0) {
      const size_t ogm = oglob(B, m, slot_at(B, m, cm_[c]));
      cs = cos_max_warp(B, ogm, B.objs[ogm], B.mu + ogn * B.D);
    }
    if (lane == 0) ccos_[c] = cs;
    __syncwarp();
  }
  __syncthreads();
  if (tid != 0) return;
  np_ = 0;
  for (int c = 0; c < cn_; ++c) {
    if (ccos_[c] < -2.5 || ccos_[c] < P.link_cos) continue;
    pd_[np_] = cd_[c];
    pm_[np_] = obj_at(B, m, cm_[c]).id;
    pn_[np_] = obj_at(B, m, cnn_[c]).id;
    ++np_;
  }
  // sort (d, mid, nid) ascending
  for (int i = 1; i < np_; ++i) {
    const double d = pd_[i];
    const uint32_t a = pm_[i], b = pn_[i];
    int j = i;
    while (j > 0 && (pd_[j - 1] > d || (pd_[j - 1] == d && (pm_[j - 1] > a || (pm_[j - 1] == a && pn_[j - 1] > b))))) {
      pd_[j] = pd_[j - 1]; pm_[j] = pm_[j - 1]; pn_[j] = pn_[j - 1];
      --j;
    }
    pd_[j] = d; pm_[j] = a; pn_[j] = b;
  }
  uint32_t used[2 * RELINK_MAXC];
  int nused = 0;
  for (int p = 0; p < np_; ++p) {
    bool u = false;
    for (int q = 0; q < nused; ++q) u = u || used[q] == pm_[p] || used[q] == pn_[p];
    if (u) continue;
    used[nused++] = pm_[p];
    used[nused++] = pn_[p];
    const int mi = find_pos(B, m, pm_[p]), ni = find_pos(B, m, pn_[p]);
    if (mi < 0 || ni < 0) continue;
    ObjRec& mo = B.objs[oglob(B, m, slot_at(B, m, mi))];
    const ObjRec& no = B.objs[oglob(B, m, slot_at(B, m, ni))];
    for (int k = 0; k < 3; ++k) { mo.pos[k] = no.pos[k]; mo.ext[k] = no.ext[k]; mo.lo[k] = no.lo[k]; mo.hi[k] = no.hi[k]; }
    // m takes n's cloud (m.cloud = n.cloud; version = n.version + 1); m's old cloud slot is freed
    if (!INB(R->n_cfree, B.C, 505)) continue;
    B.cfreel[(size_t)m * B.C + R->n_cfree++] = mo.cloud_slot;
    mo.cloud_slot = no.cloud_slot;
    ++B.clouds[cglob(B, m, mo.cloud_slot)].version;
    mo.n_obs += no.n_obs;
    mo.last_seen = no.last_seen;
    mo.last_kf = no.last_kf;
    mo.score = (mo.score < no.score) ? no.score : mo.score;
    mo.max_det_z = smax(mo.max_det_z, no.max_det_z);
    for (int k = 0; k < 3; ++k) mo.trk_pos[k] = no.trk_pos[k];
    mo.trk_t = no.trk_t;
    mo.mv_cnt = 0;
    mo.appeared = 0;
    mo.moved = 1;
    mo.state = 2;
    mo.misses = 0;
    mo.parent = 0;
    remap_id(B, m, pn_[p], pm_[p]);
    push_event(B, m, t, mo, 2, (4u << 24) | (uint32_t)p);
    erase_pos(B, m, ni, true);
  }
}

// apStructObject geometry (objmap.cpp:1255-1319) for objects whose cloud changed; no wall
// segments and no text model, so only geo 1 (wall-size vertical plane) / 2 (ceiling) matter.
#define STRUCT_PTS 1600   // cloudSample(800) keeps ceil(n / max(1, n / 800)) < 1600 points
#define STRUCT_SMEM (sizeof(PlaneSmem) + 3 * STRUCT_PTS * sizeof(float))   // dynamic: plane-fit working set + sample
__global__ void __launch_bounds__(256, 4) k_struct(Batch B) {
  extern __shared__ __align__(16) unsigned char st_raw[];
  PlaneSmem& ps = *(PlaneSmem*)st_raw;
  float* Pt = (float*)(st_raw + sizeof(PlaneSmem));   // cloudSample(800) points (shared)
  __shared__ BlockScratch bs;
  __shared__ PlaneOut pout;
  __shared__ int mine[STRUCT_LIST];
  __shared__ int nmine;
  __shared__ int scan_db[2][33];
  const int m = B.map0 + blockIdx.y;
  const FrameDev& F = B.frames[m];
  if (!F.active) return;
  const MapRec& R = B.maps[m];
  const smg_params& P = B.p;
  double* sel = B.sscr + ((size_t)m * gridDim.x + blockIdx.x) * STRUCT_SCR;
  double* scr = sel + 4096;                 // plane-fit scratch: 2 x 4096 doubles
  // the objects whose cloud changed, in list order; CTA c takes every gridDim.x-th of them
  if (threadIdx.x == 0) nmine = 0;
  int before = 0, it = 0;
  for (int c0 = 0; c0 < R.n_obj; c0 += blockDim.x) {
    const int b = c0 + threadIdx.x;
    int need = 0;
    if (b < R.n_obj) {
      const ObjRec& o = B.objs[oglob(B, m, slot_at(B, m, b))];
      const CloudRec& C = B.clouds[cglob(B, m, o.cloud_slot)];
      need = o.held_by < 0 && o.geo_ver != C.version && C.n >= 30;
    }
    int tot;
    const int rank = before + block_scan_db(need, &tot, scan_db, it++);
    if (need && rank % (int)gridDim.x == (int)blockIdx.x) {
      const int q = atomicAdd(&nmine, 1);
      if (q < STRUCT_LIST) mine[q] = b;
    }
    before += tot;
  }
  __syncthreads();
  const int nm = nmine < STRUCT_LIST ? nmine : STRUCT_LIST;
  if (threadIdx.x == 0 && nmine > STRUCT_LIST) set_err(&B.maps[m], SMG_E_ARGS);
  // the list came out of an unordered append; objects are independent, so order is free
  for (int q = 0; q < nm; ++q) {
    const int b = mine[q];
    ObjRec& o = B.objs[oglob(B, m, slot_at(B, m, b))];
    const size_t cs = cglob(B, m, o.cloud_slot);
    const CloudRec& C = B.clouds[cs];
    // cloudSample(m, 800) (objmap.cpp:1107-1114)
    const size_t stp = (size_t)C.n / 800 > 1 ? (size_t)C.n / 800 : 1;
    const int n = (int)(((size_t)C.n + stp - 1) / stp);
    const float4* pts = B.cpts + cs * B.cap;
    if (!INB(n, STRUCT_PTS, 508)) continue;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const float4 qp = pts[(size_t)i * stp];
      Pt[3 * i] = (float)(C.org[0] + (double)qp.x);
      Pt[3 * i + 1] = (float)(C.org[1] + (double)qp.y);
      Pt[3 * i + 2] = (float)(C.org[2] + (double)qp.z);
    }
    __syncthreads();
    plane_fit(Pt, n, P.obj_tau, ap_seed((uint64_t)o.id, (uint64_t)C.version), P.ransac_iters, B.need_tab, scr, 4096, &ps, bs,
              &pout, 12);
    int up = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) up += (double)Pt[3 * i + 2] > R.ceil_est - P.ceil_band;
    up = block_sum_i(up, bs);
    // wall lines (ObjectMap::wsegs_): points within wall_d (the share fw, objmap.cpp:1298-1302)
    // and within obj_flat_d (the flat-plane test, :1310-1317) of some stored segment
    const bool walls = R.n_wseg > 0;
    int nw = 0, nflat = 0;
    if (walls && n > 0) {
      const double* S = B.wsegs + (size_t)m * SMG_WALL_SEGS_MAX * 4;
      const double stop = smin(P.wall_d, P.obj_flat_d);
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const double dm = wall_dist((double)Pt[3 * i], (double)Pt[3 * i + 1], S, R.n_wseg, stop);
        nw += dm <= P.wall_d;
        nflat += dm <= P.obj_flat_d;
      }
      nw = block_sum_i(nw, bs);
      nflat = block_sum_i(nflat, bs);
    }
    if (threadIdx.x == 0) {
      o.geo_ver = C.version;
      int geo = 0;
      const double nz = fabs(pout.n[2]);
      const bool plane = pout.ok && pout.inl >= P.obj_plane_inl;
      if (plane && pout.thick < P.obj_thick) {
        if (nz < P.wall_vert && (pout.hspan >= P.obj_wall_span || (pout.zhi >= P.obj_wall_top && pout.zhi - pout.zlo >= P.obj_wall_h))) geo = 1;
        else if (nz > P.horiz && pout.zmed > P.ceil_z) geo = 2;
      }
      if (!geo && R.ceil_est > 0 && n > 0)
        if (up >= P.ceil_frac * n && smax(o.hi[0] - o.lo[0], o.hi[1] - o.lo[1]) >= P.ceil_wide) geo = 2;
      o.fw = n > 0 ? (float)((double)nw / n) : 0.f;
      // a very thin upright plane on a wall line: door leaf, window pane (objmap.cpp:1310-1317)
      if (!geo && plane && pout.thick < P.obj_flat_thick && nz < P.wall_vert && walls && n > 0 && !(nflat < P.obj_flat_frac * n))
        geo = 3;
      o.geo = geo;
      o.vinl = pout.ok && nz < P.wall_vert ? (float)pout.inl : 0.f;
    }
    __syncthreads();
    if ((B.text_on || walls) && n > 0) {
      // the shape the named-structure and wall-hugging rules read (objmap.cpp:1281-1301): 5-95 %
      // spans along the horizontal principal axes and in height.  Without a text model and
      // without wall segments no rule reads it (fw is then 0).
      double sx = 0, sy = 0;
      for (int i = threadIdx.x; i < n; i += blockDim.x) { sx += (double)Pt[3 * i]; sy += (double)Pt[3 * i + 1]; }
      const double mx = block_sum_d(sx, bs) / n, my = block_sum_d(sy, bs) / n;
      double a3[3] = {0, 0, 0};
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const double dx = (double)Pt[3 * i] - mx, dy = (double)Pt[3 * i + 1] - my;
        a3[0] += dx * dx; a3[1] += dx * dy; a3[2] += dy * dy;
      }
      __shared__ double red3[3 * 32];
      block_sum_multi<3>(a3, red3);
      const double th = 0.5 * atan2(2 * a3[1], a3[0] - a3[2]), c = cos(th), sn = sin(th);
      double* U = scr;
      double* V = scr + STRUCT_PTS;
      double* Z = scr + 2 * STRUCT_PTS;
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const double dx = (double)Pt[3 * i] - mx, dy = (double)Pt[3 * i + 1] - my;
        U[i] = dx * c + dy * sn;
        V[i] = -dx * sn + dy * c;
        Z[i] = (double)Pt[3 * i + 2];
      }
      __syncthreads();
      int* hist = (int*)Pt;   // the sample is dead: selection histograms
      __shared__ double sel6[6];
      const double* arr[6] = {U, U, V, V, Z, Z};
      const int nn[6] = {n, n, n, n, n, n};
      const int k5 = pct_index(n, 0.05), k95 = pct_index(n, 0.95);
      const int kk[6] = {k95, k5, k95, k5, k95, k5};
      block_select_multi(arr, nn, kk, sel6, 6, hist, bs);
      if (threadIdx.x == 0) {
        const double su = sel6[0] - sel6[1], sv = sel6[2] - sel6[3];
        o.maj = (double)(float)smax(su, sv);
        o.minr = (double)(float)smin(su, sv);
        o.hgt = (double)(float)(sel6[4] - sel6[5]);
      }
      __syncthreads();
    }
  }
}

// apStructObject's decision (objmap.cpp:1320-1349) on the object's geometry, wall share and
// name posterior; sets hide.
DEV bool struct_object_drop(const Batch& B, size_t og, ObjRec& o) {
  const smg_params& P = B.p;
  o.hide = 0;
  const int C = B.txt.n_labels;
  const float* post = o.has_post ? B.post + og * C : nullptr;
  double qso = 0;
  if (post)
    for (int l = 0; l < C; ++l)
      if (kind_of(B, l) == KIND_STRUCT_OBJ) qso += (double)post[l];
  const double fw = (double)o.fw;
  if (qso >= 0.5 && o.geo != 2) {
    double qsh[4] = {0, 0, 0, 0};
    for (int l = 0; l < C; ++l)
      if (kind_of(B, l) == KIND_STRUCT_OBJ) qsh[B.txt.so_shape ? B.txt.so_shape[l] & 3 : 0] += (double)post[l];
    int sh = 1;
    for (int i = 2; i < 4; ++i)
      if (qsh[i] > qsh[sh]) sh = i;
    const bool fits = sh == 1   ? o.maj <= P.so_dw_w && o.minr <= P.so_dw_thick && o.hgt <= P.so_max_h
                      : sh == 3 ? o.maj <= P.so_pillar
                                : o.maj <= P.so_stairs;
    if (sh == 1 && o.maj < P.so_dw_min && (int)o.n_obs >= P.so_min_obs) return true;
    if (fits) return false;
    const double lim = sh == 1 ? P.so_dw_w : sh == 3 ? P.so_pillar : P.so_stairs;
    o.hide = o.geo != 0 || (fw >= P.wallhug_frac && o.maj >= P.wallhug_w) || (double)o.vinl >= P.big_vinl || o.maj > P.so_hide_k * lim;
    return false;
  }
  if (flat_named(B, o) && o.maj > P.flat_max_w && (o.geo != 0 || fw >= 0.5 || (double)o.vinl >= P.big_vinl)) { o.hide = 1; return false; }
  if (fw >= P.wallhug_frac && o.maj >= P.wallhug_w) { o.hide = 1; return false; }
  if (o.geo == 3) {   // a flat plane on a wall line stays only under a flat-object or structural-object name
    double q = qso;
    if (post && B.txt.flat_ok)
      for (int l = 0; l < C; ++l)
        if (B.txt.flat_ok[l]) q += (double)post[l];
    if (q < P.flat_keep_p) return true;
  }
  if (o.geo == 1 || o.geo == 2) return true;
  if (o.n_whole < P.struct_obj_min_views || !post) return false;
  double q = 0;
  for (int l = 0; l < C; ++l)
    if (kind_of(B, l) == KIND_STRUCTURE) q += (double)post[l];
  return q >= P.struct_obj_p;
}

// drop + prune (objmap.cpp:1064-1073), then the cloud-addition targets (objects named by this
// frame's cloud lists, first appearance order, plus objects whose cloud moved).  The list is
// staged in shared memory; removal flags are evaluated in parallel, the ordered compaction and
// the target list by thread 0.
#define PRUNE_MAX 4096
__global__ void __launch_bounds__(256) k_prune(Batch B) {
  __shared__ int s_slot[PRUNE_MAX];
  __shared__ uint32_t s_id[PRUNE_MAX];
  __shared__ unsigned char s_rm[PRUNE_MAX], s_dirty[PRUNE_MAX], s_fe[PRUNE_MAX];
  __shared__ BlockScratch bs;
  const int m = B.map0 + blockIdx.x, tid = threadIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active) return;
  MapRec* R = &B.maps[m];
  const smg_params& P = B.p;
  const int n = R->n_obj;
  if (n > PRUNE_MAX) {
    if (tid == 0) set_err(R, SMG_E_CAP_OBJ);
    return;
  }
  int nstruct = 0;
  for (int b = tid; b < n; b += blockDim.x) {
    const int slot = slot_at(B, m, b);
    ObjRec& o = B.objs[oglob(B, m, slot)];
    if (o.held_by >= 0) {   // apStructObject returns false for a held object (objmap.cpp:1256)
      o.drop = 0;
    } else {
      o.drop = struct_object_drop(B, oglob(B, m, slot), o);
    }
    bool rm;
    if (o.drop) { ++nstruct; rm = true; }
    else if (!o.confirmed) rm = F.stamp - o.last_seen > P.prune_s;
    else rm = o.state == 1 && !o.moved && (int)o.n_obs < P.spurious_obs;
    const CloudRec& C = B.clouds[cglob(B, m, o.cloud_slot)];
    s_slot[b] = slot;
    s_id[b] = o.id;
    s_rm[b] = rm;
    s_dirty[b] = C.cver != C.version && C.n > 0;
  }
  nstruct = block_sum_i(nstruct, bs);
  // everything below is list-ordered compaction, done with block scans: kept objects to the
  // list, removed ones to the free lists (in list order), then the cloud targets
  const int nfree0 = R->n_free, ncfree0 = R->n_cfree, npts = min(R->n_pts, B.max_det);
  __shared__ uint32_t s_pid[SMG_MAX_DET];
  __shared__ int s_byE[SMG_MAX_DET];
  __shared__ int pr_db[2][33];
  for (int e = tid; e < npts; e += blockDim.x) { s_pid[e] = B.ptsl[(size_t)m * B.max_det + e].obj_id; s_byE[e] = -1; }
  __syncthreads();
  int32_t* ord = B.order + (size_t)m * B.O;
  int it = 0, kept = 0, rmd = 0;
  for (int c0 = 0; c0 < n; c0 += blockDim.x) {
    const int b = c0 + tid;
    const int rm = b < n && s_rm[b], keep = b < n && !s_rm[b];
    int tk, tr;
    const int pk = block_scan_db(keep, &tk, pr_db, it++);
    const int pr = block_scan_db(rm, &tr, pr_db, it++);
    if (keep) {
      ord[kept + pk] = s_slot[b];
      // first cloud list of this object (each list names one object)
      int fe = 255;
      for (int e = 0; e < npts; ++e)
        if (s_pid[e] == s_id[b]) { fe = e; break; }
      s_fe[b] = (unsigned char)fe;
      if (fe < 255) s_byE[fe] = b;
    }
    if (rm) {
      const ObjRec& o = B.objs[oglob(B, m, s_slot[b])];
      if (INB(ncfree0 + rmd + pr, B.C, 510)) B.cfreel[(size_t)m * B.C + ncfree0 + rmd + pr] = o.cloud_slot;
      if (INB(nfree0 + rmd + pr, B.O, 511)) B.freel[(size_t)m * B.O + nfree0 + rmd + pr] = s_slot[b];
    }
    kept += tk;
    rmd += tr;
  }
  __syncthreads();
  // targets: the objects of the cloud lists in list order, then the kept objects whose contact
  // index is stale, in object-list order
  int32_t* TG = B.tgt_slot + (size_t)m * B.O;
  __shared__ int s_na;
  if (tid == 0) {
    int na = 0;
    for (int e = 0; e < npts; ++e)
      if (s_byE[e] >= 0) TG[na++] = s_slot[s_byE[e]];
    s_na = na;
  }
  __syncthreads();
  int nt = s_na;
  for (int c0 = 0; c0 < n; c0 += blockDim.x) {
    const int b = c0 + tid;
    const int f = b < n && !s_rm[b] && s_dirty[b] && s_fe[b] == 255;
    int tot;
    const int pos = block_scan_db(f, &tot, pr_db, it++);
    if (f && INB(nt + pos, B.O, 512)) TG[nt + pos] = s_slot[b];
    nt += tot;
  }
  if (tid == 0) {
    R->st.n_obj_struct += nstruct;
    R->n_cfree = ncfree0 + rmd <= B.C ? ncfree0 + rmd : B.C;
    R->n_free = nfree0 + rmd <= B.O ? nfree0 + rmd : B.O;
    R->n_obj = kept;
    R->n_targets = nt;
  }
}

// markView (objmap.cpp:219-245): sparse depth samples, horizontal camera->point segments, first
// time each 2D cell was seen per range band.  Fresh cells are pre-filled with "never".
#define MV_CTAS 24    // k_markview CTAs per map
#define MV_SPLIT 8    // threads per sampled pixel: each marches every MV_SPLIT-th step of its ray
__global__ void __launch_bounds__(256) k_markview(Batch B) {
  const int m = B.map0 + blockIdx.y;
  const FrameDev& F = B.frames[m];
  if (!F.active) return;
  const smg_params& P = B.p;
  const double* T = F.T_mc;
  const double cell = smax(0.05, P.view_cell);
  const int stp = max(1, F.w / 32);
  const int nu = (F.w - stp / 2 + stp - 1) / stp, nv = (F.h - stp / 2 + stp - 1) / stp;
  int64_t* K = B.vkey + (size_t)m * B.view_slots;
  // the view cells a ray covers and their first stamps do not depend on the order of the steps
  // (every write of the frame stores the same stamp), so the steps are split across threads
  for (int g = blockIdx.x * blockDim.x + threadIdx.x; g < nu * nv * MV_SPLIT; g += gridDim.x * blockDim.x) {
    const int s = g / MV_SPLIT, j = g - s * MV_SPLIT;
    const int u = stp / 2 + (s % nu) * stp, v = stp / 2 + (s / nu) * stp;
    const float z = F.depth[(size_t)v * F.w + u];
    if (!(z > P.zmin && z < P.zmax)) continue;
    const double xc = (double)(((float)u - F.cx) / F.fx * z), yc = (double)(((float)v - F.cy) / F.fy * z);
    const double zd = (double)z;
    const double px = T[0] * xc + T[1] * yc + T[2] * zd + T[3];
    const double py = T[4] * xc + T[5] * yc + T[6] * zd + T[7];
    const double dx = px - T[3], dy = py - T[7];
    const double L = sqrt(dx * dx + dy * dy), Lm = smin(L, (double)SMG_VIEW_BANDS);
    if (L < 1e-6) continue;
    const int ns = (int)ceil(Lm / (0.5 * cell));
    for (int q = j; q <= ns; q += MV_SPLIT) {
      const double r = Lm * q / (double)max(1, ns);
      const int64_t key = view_cell_key(T[3] + r / L * dx, T[7] + r / L * dy, cell);
      uint32_t h = hmix((uint64_t)key) & (uint32_t)(B.view_slots - 1);
      int probe = 0;
      for (; probe < B.view_slots; ++probe) {
        const unsigned long long prev =
            atomicCAS((unsigned long long*)&K[h], (unsigned long long)INT64_MIN, (unsigned long long)key);
        if (prev == (unsigned long long)INT64_MIN || prev == (unsigned long long)key) break;
        h = (h + 1) & (uint32_t)(B.view_slots - 1);
      }
      if (probe == B.view_slots) { set_err(&B.maps[m], SMG_E_CAP_VIEW); continue; }
      double* e = B.vfirst + ((size_t)m * B.view_slots + h) * SMG_VIEW_BANDS;
      for (int b = max(0, (int)ceil(r) - 1); b < SMG_VIEW_BANDS; ++b)
        if (e[b] < -1e299) e[b] = F.stamp;
    }
  }
}
