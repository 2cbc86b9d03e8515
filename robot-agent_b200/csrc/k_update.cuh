// Object update of one keyframe (scenemap src/objmap.cpp:807-1019) in two kernels.
//
// The reference's update is a sequence over observations whose later steps depend on the
// earlier ones (fragments fuse into the first, largest one; new objects are appended mid-loop
// and can capture later fragments).  k_update keeps that order where it matters: one CTA per
// map; thread 0 walks the observations for the decisions that cross objects (actions, slots and
// ids, frame grouping, job places, event numbers), and each staged object then applies its own
// observations in order on its own thread (the scalar half of apAddView -- tempering, camera
// ring, view list -- and the Kalman/tracking/state update), recording each embedding's D-length
// work as a job.
// k_update_vec then runs one CTA per target object and applies its jobs in observation order
// (r_frag += k z in fp32, the fp16 view copy, |r_frag|^2 and mu); the objects are independent.
// The frame-grouping dot products were computed by k_assoc.
#pragma once
#include "k_assoc.cuh"

#define UPD_THREADS 256
#define UPD_SMEM(B) ((size_t)(B).max_det * (sizeof(ObsRec) + sizeof(ObjRec)))

// one warp copies an object record in 16-byte words, all of a lane's loads issued first
static_assert(sizeof(ObjRec) % 16 == 0, "ObjRec is copied in 16-byte words");
DEV void rec_load(ObjRec* dst, const ObjRec* src) {
  constexpr int NW = (int)(sizeof(ObjRec) / 16), PER = (NW + 31) / 32;
  const int lane = threadIdx.x & 31;
  const uint4* s = (const uint4*)src;
  uint4* d = (uint4*)dst;
  uint4 t[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j)
    if (j * 32 + lane < NW) t[j] = s[j * 32 + lane];
#pragma unroll
  for (int j = 0; j < PER; ++j)
    if (j * 32 + lane < NW) d[j * 32 + lane] = t[j];
}

DEV size_t cslot_glob(const Batch& B, int m, const ObjRec& o) { return cglob(B, m, o.cloud_slot); }

// ObjectMap::firstView (objmap.cpp:247-252) over the view-first hash
DEV int64_t view_cell_key(double x, double y, double cell) {
  const long long i = (long long)floor(x / cell), j = (long long)floor(y / cell);
  return (int64_t)(((unsigned long long)i << 32) ^ ((unsigned long long)j & 0xffffffffull));
}
DEV double first_view(const Batch& B, int m, double x, double y, double range) {
  const double cell = smax(0.05, B.p.view_cell);
  const int64_t key = view_cell_key(x, y, cell);
  const int64_t* K = B.vkey + (size_t)m * B.view_slots;
  uint32_t h = hmix((uint64_t)key) & (uint32_t)(B.view_slots - 1);
  for (int probe = 0; probe < B.view_slots; ++probe) {
    if (K[h] == INT64_MIN) return 1e300;
    if (K[h] == key) {
      int b = (int)ceil(range) - 1;
      b = b < 0 ? 0 : (b > SMG_VIEW_BANDS - 1 ? SMG_VIEW_BANDS - 1 : b);
      const double v = B.vfirst[((size_t)m * B.view_slots + h) * SMG_VIEW_BANDS + b];
      return v < -1e299 ? 1e300 : v;
    }
    h = (h + 1) & (uint32_t)(B.view_slots - 1);
  }
  return 1e300;
}

// |r_frag|^2 and the mean direction mu = float(r / |r|) (ApState mu cache, objprob.cpp:228-240),
// block-wide, after every change of r_frag
// apCache (objprob.cpp:228-240): |r_frag|^2, |r_whole|^2 and mu = the whole vector's direction
// when the object has whole-view weight (k_whole > 0), else the fragment sum's.  Block-wide;
// the norms go to record `o` (a staged copy or the object itself).
DEV void refresh_nrm_into(const Batch& B, ObjRec& o, size_t og, BlockScratch& bs) {
  const float* rf = B.rfrag + og * B.D;
  const float* rw = B.rwhole + og * B.D;
  const bool hw = o.has_whole != 0;
  double s = 0, sw = 0;
  for (int i = threadIdx.x; i < B.D; i += blockDim.x) {
    s += (double)rf[i] * (double)rf[i];
    if (hw) sw += (double)rw[i] * (double)rw[i];
  }
  s = block_sum_d(s, bs);
  sw = hw ? block_sum_d(sw, bs) : 0.0;
  const bool use_w = o.k_whole > 0;
  __syncthreads();
  if (threadIdx.x == 0) { o.nrm_frag = s; o.nrm_whole = sw; }
  const float* r = use_w ? rw : rf;
  const double n2 = use_w ? sw : s, nn = sqrt(n2);
  float* mu = B.mu + og * B.D;
  for (int i = threadIdx.x; i < B.D; i += blockDim.x) mu[i] = n2 > 0 ? (float)((double)r[i] / nn) : 0.f;
  __syncthreads();
}
DEV void refresh_nrm(const Batch& B, size_t og, BlockScratch& bs) { refresh_nrm_into(B, B.objs[og], og, bs); }

// apAddView (scenemap objprob.cpp:312-356), no text model: the scalar part, run by one thread -- view tempering against the camera ring
// (similar view at another stamp: kappa * temper), the ring of the newest 32 cameras, ver and
// k_frag, the physical view slot the fp16 copy goes to and the view list kept sorted by kappa
// (stable, top-k).  The D-length part (r_frag += k z, the fp16 copy, |r|^2, mu) is recorded as
// a job for k_update_vec.
DEV void ap_add_view_plan(const Batch& B, ObjRec& o, double kappa, double stamp, const double cam[6], double* k_out, int* phys_out,
                          bool whole = false) {
  double k = kappa;
  const double cmin = B.cos_temper;
  const double td = B.p.temper_d, td2 = td * td;
  for (int c = 0; c < o.n_cams; ++c) {
    const double* cc = cam_at(o, c);
    if (fabs(cc[6] - stamp) < 1e-6) continue;
    const double ca = cc[3] * cam[3] + cc[4] * cam[4] + cc[5] * cam[5];
    if (!(ca > cmin)) continue;
    // hypot(d) < temper_d: the squared norm decides it unless it lies within rounding of the
    // bound, where the 3-argument hypot itself is evaluated
    const double dx = cc[0] - cam[0], dy = cc[1] - cam[1], dz = cc[2] - cam[2];
    const double s2 = dx * dx + dy * dy + dz * dz;
    const bool close = fabs(s2 - td2) <= 1e-12 * td2 ? hypot3(dx, dy, dz) < td : s2 < td2;
    if (close) { k = kappa * B.p.temper; break; }
  }
  {   // keep the newest 32 (push, then erase the front)
    const double c7[7] = {cam[0], cam[1], cam[2], cam[3], cam[4], cam[5], stamp};
    cam_push(o, c7);
  }
  ++o.ver;
  if (whole) {
    o.k_whole += k;
    ++o.n_whole;
    o.whole_kappa = smax(o.whole_kappa, kappa);
    o.need_whole = 0;
  } else {
    o.k_frag += k;
  }
  // free physical view slot: the one of 0..topk not referenced by the current views
  int used = 0;
  for (int v = 0; v < o.n_views; ++v) if (INB(o.view_slot[v], B.topk + 1, 301)) used |= 1 << o.view_slot[v];
  int f = 0;
  while (used & (1 << f)) ++f;
  // stable sort by (whole desc, kappa desc): the new view goes after every view that is whole
  // while it is not, or of its own kind with a kappa >= its own; then keep the top-k
  const float kv = (float)kappa;
  const int wv = whole ? 1 : 0;
  int pos = o.n_views;
  while (pos > 0 && (o.vwhole[pos - 1] < wv || (o.vwhole[pos - 1] == wv && o.vkappa[pos - 1] < kv))) --pos;
  for (int v = o.n_views; v > pos; --v) {
    o.view_slot[v] = o.view_slot[v - 1];
    o.vkappa[v] = o.vkappa[v - 1];
    o.vstamp[v] = o.vstamp[v - 1];
    o.vwhole[v] = o.vwhole[v - 1];
  }
  o.view_slot[pos] = f;
  o.vkappa[pos] = kv;
  o.vstamp[pos] = stamp;
  o.vwhole[pos] = wv;
  ++o.n_views;
  if (o.n_views > B.topk) o.n_views = B.topk;
  *k_out = k;
  *phys_out = f;
}

// push_event with the map's event count held by the caller (ev_base at entry, *evl added since)
DEV void push_event_l(const Batch& B, int map, double t, const ObjRec& o, int kind, uint32_t key, int ev_base, int* evl) {
  const int e = ev_base + (*evl)++;
  if (e >= SMG_MAX_EVENTS) { set_err(&B.maps[map], SMG_E_CAP_EVENTS); return; }
  EventRec& r = B.events[(size_t)map * SMG_MAX_EVENTS + e];
  r.t = t;
  r.id = o.id;
  r.kind = kind;
  r.key = key;
}


__global__ void __launch_bounds__(UPD_THREADS) k_update(Batch B) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  ObjRec* REC = (ObjRec*)smem_raw;                 // staged object records, indexed by observation
  ObsRec* OB = (ObsRec*)(REC + B.max_det);         // staged observations
  __shared__ int OL[SMG_MAX_DET];                  // observation list (detection order)
  __shared__ int rec_slot[SMG_MAX_DET];            // object slot of record a (-1: record unused)
  __shared__ int obs_rec[SMG_MAX_DET];             // record of each listed observation (-1: none)
  __shared__ int head[SMG_MAX_DET];
  __shared__ int fl[SMG_MAX_DET], cfl[SMG_MAX_DET];   // the free-list entries new objects pop, in order
  __shared__ int64_t tg_og[SMG_MAX_DET];           // target objects of the vector jobs
  __shared__ int n_book[3], njobs, ntg;
  const int m = B.map0 + blockIdx.x, tid = threadIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active) return;
  MapRec* R = &B.maps[m];
  const smg_params& P = B.p;
  const double* T = F.T_mc;
  const int nobs = R->n_obs, n_obj0 = R->n_obj, n_free0 = R->n_free, n_cfree0 = R->n_cfree;
  const bool has_z = F.emb != nullptr;
  {
    const uint32_t* src = (const uint32_t*)(B.obs + (size_t)m * B.max_det);
    uint32_t* dst = (uint32_t*)OB;
    for (int i = tid; i < (int)(B.max_det * sizeof(ObsRec) / 4); i += blockDim.x) dst[i] = src[i];
    for (int i = tid; i < nobs; i += blockDim.x) OL[i] = B.obs_list[(size_t)m * B.max_det + i];
    if (tid < 3) n_book[tid] = 0;
  }
  const double* GD = B.gdot + (size_t)m * B.max_det * B.max_det;
  const double cam6[6] = {T[3], T[7], T[11], T[2], T[6], T[10]};
  __syncthreads();
  // association bookkeeping (objmap.cpp:807-809), one thread per observation
  if (tid < nobs) {
    ObsRec& o = OB[OL[tid]];
    if (P.bridge_drop && o.n_same >= 2 && o.obs_to >= 0) { o.obs_to = -2; atomicAdd(&n_book[0], 1); }
    else if (o.obs_to >= 0) { B.obj_hit[(size_t)m * B.O + o.obs_to] = 1; atomicAdd(&n_book[1], 1); }
    else if (o.blocked) { o.obs_to = -2; atomicAdd(&n_book[2], 1); }
  }
  __syncthreads();
  // per observation: its fusion head (the first fragment of its target with the most points,
  // objmap.cpp:812-820) and its staged record (the target's first observation)
  if (tid < nobs) {
    const int b = OB[OL[tid]].obs_to;
    int h = -1, first = -1;
    if (b >= 0)
      for (int a2 = 0; a2 < nobs; ++a2) {
        const ObsRec& q = OB[OL[a2]];
        if (q.obs_to != b) continue;
        if (first < 0) first = a2;
        if (h < 0 || q.n > OB[OL[h]].n) h = a2;
      }
    head[tid] = h;
    const bool valid = b >= 0 && INB(b, n_obj0, 302);
    obs_rec[tid] = valid ? first : -1;
    rec_slot[tid] = valid && first == tid ? slot_at(B, m, b) : -1;
    fl[tid] = tid < n_free0 && INB(n_free0 - 1 - tid, B.O, 303) ? B.freel[(size_t)m * B.O + n_free0 - 1 - tid] : -1;
    cfl[tid] = tid < n_cfree0 && INB(n_cfree0 - 1 - tid, B.C, 303) ? B.cfreel[(size_t)m * B.C + n_cfree0 - 1 - tid] : -1;
  }
  __syncthreads();
  for (int r = tid >> 5; r < nobs; r += blockDim.x >> 5)
    if (rec_slot[r] >= 0) rec_load(&REC[r], &B.objs[oglob(B, m, rec_slot[r])]);
  __syncthreads();
  // The per-observation walk below runs on thread 0 against the staged copies, with the map
  // scalars in registers: it waits on no global load.
  uint32_t next_id = 0;
  int n_obj = n_obj0, n_free = n_free0, n_cfree = n_cfree0, n_pop = 0, evn = 0, evl = 0, ev_base = 0;
  long long n_new = 0;
  if (tid == 0) {
    next_id = R->next_id;
    ev_base = R->n_events;
    njobs = 0;
    ntg = 0;
    // fragment fusion (objmap.cpp:821-835) into each head, in observation order
    for (int a = 0; a < nobs; ++a) {
      ObsRec& o = OB[OL[a]];
      const int b = o.obs_to;
      if (b < 0 || head[a] == a) continue;
      ObsRec& h = OB[OL[head[a]]];
      const double wh = h.n, wo = o.n;
      for (int k = 0; k < 3; ++k) {
        h.lo[k] = smin(h.lo[k], o.lo[k]);
        h.hi[k] = smax(h.hi[k], o.hi[k]);
        h.pos[k] = (h.pos[k] * wh + o.pos[k] * wo) / (wh + wo);
        h.ext[k] = h.hi[k] - h.lo[k];
      }
      h.n += o.n;
      h.trunc = h.trunc || o.trunc;
      h.zmed = smin(h.zmed, o.zmed);
      h.score = (h.score < o.score) ? o.score : h.score;
      o.sec = 1;
    }
  }
  // update loop (objmap.cpp:837-997), in three steps.  P1 (thread 0, observation order): the
  // association record, the action (update a staged object or create one), slot and id
  // allocation, the frame grouping of later fragments and the vector jobs' places.  P2 (one
  // thread per staged record, its observations in order): the object's own update -- the
  // scalar half of apAddView, Kalman, tracking, state -- which reads and writes no other
  // object.  P3 (thread 0): the events, numbered in observation order.
  __shared__ signed char s_act[SMG_MAX_DET], s_evf[SMG_MAX_DET];
  __shared__ int s_job[SMG_MAX_DET], s_cs[SMG_MAX_DET];
  __shared__ uint32_t s_newid[SMG_MAX_DET];
  const size_t jbase = (size_t)m * B.max_det;
  if (tid == 0) {
    for (int a = 0; a < nobs; ++a) {
      ObsRec& o = OB[OL[a]];
      AssocRec& as = B.assoc[(size_t)m * B.max_det + o.det];
      as.n_valid = o.n;
      as.area_px = (float)o.n * o.sk * o.sk;
      as.depth_med = (float)o.zmed;
      int act = 0, r = -1;
      s_evf[a] = 0;
      s_job[a] = -1;
      if (o.obs_to >= 0 && INB(o.obs_to, n_obj, 302) && obs_rec[a] >= 0) {
        act = 1;
        r = obs_rec[a];
        as.obj_id = s_act[r] == 2 && r < a ? s_newid[r] : REC[r].id;   // a grouped fragment's object is built in P2
      } else if (o.obs_to == -1) {   // ObjectMap slot allocation (new object)
        if (n_free <= 0 || n_cfree <= 0 || n_obj >= B.O || !INB(n_pop, nobs, 303) || fl[n_pop] < 0 || cfl[n_pop] < 0) {
          set_err(R, SMG_E_CAP_OBJ);
        } else {
          const int slot = fl[n_pop];
          s_cs[a] = cfl[n_pop];
          ++n_pop;
          --n_free;
          --n_cfree;
          B.order[(size_t)m * B.O + n_obj++] = slot;
          act = 2;
          r = a;   // an unmatched observation's own record is free
          rec_slot[r] = slot;
          obs_rec[a] = r;
          s_newid[a] = next_id++;
          as.obj_id = s_newid[a];
          B.touched[(size_t)m * B.O + n_obj - 1] = 1;
          B.obj_hit[(size_t)m * B.O + n_obj - 1] = 1;
          ++n_new;
          // frame grouping (objmap.cpp:980-995): later unmatched fragments touching this one, with
          // the dot products computed by k_assoc
          if (P.frame_group) {
            for (int b2 = a + 1; b2 < nobs; ++b2) {
              ObsRec& q = OB[OL[b2]];
              if (q.obs_to != -1 || !has_z) continue;
              double g2 = 0;
              for (int k = 0; k < 3; ++k) {
                const double g = smax3(0.0, q.lo[k] - o.hi[k], o.lo[k] - q.hi[k]);
                g2 += g * g;
              }
              if (g2 > 0.02 * 0.02) continue;
              double f[7] = {0, 0, 0, 0, 0, 0, 0};
              pair_geo(q.lo, q.hi, q.pos, o.lo, o.hi, o.pos, GD[(size_t)a * B.max_det + b2], P.cos0, f);
              f[0] = 1.0;
              if (1.0 / (1.0 + exp(-same_logit(P.w, f))) >= P.same_p) { q.obs_to = n_obj - 1; obs_rec[b2] = r; }
            }
          }
        }
      }
      s_act[a] = (signed char)act;
      // the vector job's place (objmap.cpp:848, :970 -> apAddView): jobs in observation order,
      // targets numbered by first appearance; k and the view slot come in P2
      if (act && has_z) {
        const int64_t og = (int64_t)oglob(B, m, rec_slot[r]);
        int tg = -1;
        for (int c = 0; c < ntg; ++c)
          if (tg_og[c] == og) { tg = c; break; }
        if (tg < 0 && INB(ntg, B.max_det, 304)) { tg = ntg++; tg_og[tg] = og; }
        if (tg >= 0 && INB(njobs, B.max_det, 305)) {
          UpdJob& j = B.upd_job[jbase + njobs];
          j.tg = tg;
          j.det = o.det;
          j.zero = act == 2;
          s_job[a] = njobs++;
        }
      }
    }
  }
  __syncthreads();
  // P2: every staged record walks its own observations in order, one record per warp (lane 0):
  // the records' paths differ, so records sharing a warp would run one after the other
  for (int r = tid >> 5; (tid & 31) == 0 && r < nobs; r += blockDim.x >> 5) {
    if (rec_slot[r] < 0) continue;
    ObjRec& mo = REC[r];
    for (int a = 0; a < nobs; ++a) {
      const int act = s_act[a];
      if (!act || obs_rec[a] != r) continue;
      const ObsRec& o = OB[OL[a]];
      if (act == 2) {   // new candidate (objmap.cpp:951-978)
        memset(&mo, 0, sizeof(ObjRec));
        mo.held_by = -1;
        mo.name_lab = -1;
        mo.top_lab = -1;
        mo.rename = B.text_on;   // seen this keyframe (objmap.cpp:1007-1008)
        mo.id = s_newid[a];
        mo.cls = o.cls;
        for (int k = 0; k < 3; ++k) { mo.pos[k] = mo.first_pos[k] = o.pos[k]; mo.ext[k] = o.ext[k]; mo.lo[k] = o.lo[k]; mo.hi[k] = o.hi[k]; }
        mo.n_obs = 1;
        mo.first_seen = mo.last_seen = mo.last_kf = F.stamp;
        for (int k = 0; k < 3; ++k) mo.trk_pos[k] = o.pos[k];
        mo.trk_t = F.stamp;
        mo.score = o.score;
        mo.max_det_z = o.zmed;
        mo.moving_t = -1e300;
        {
          const double hx = o.pos[0] - T[3], hy = o.pos[1] - T[7];
          mo.appeared = first_view(B, m, o.pos[0], o.pos[1], sqrt(hx * hx + hy * hy) + P.view_cell) < F.stamp - P.link_view_gap_s;
        }
        mo.confirmed = P.confirm <= 1;
        mo.cloud_slot = s_cs[a];
        mo.need_whole = 1;
        mo.geo_ver = 0xffffffffu;
        const double sd = P.ap_r0 + P.ap_r1 * o.zmed;
        for (int k = 0; k < 3; ++k) mo.P[k] = sd * sd + (o.trunc ? 0.25 * o.ext[k] * o.ext[k] : 0.0);
        CloudRec& C = B.clouds[cglob(B, m, s_cs[a])];
        C.has_org = 0;
        C.n = 0;
        C.version = 0;
        C.seq = 0;
        C.stamp = 0;
        C.cn = 0;
        ++C.cgen;
        ++C.vgen;
        C.cver = 0xffffffffu;
        mo.n_ap_obs = 1;
        mo.n_wall_obs = o.wall_like;
        mo.n_struct_look = o.struct_look;
        mo.wall_like = o.wall_like;
      }
      if (has_z) {   // a recycled slot starts from an empty r_frag (objprob.cpp:329 assigns zeros)
        double k;
        int phys;
        ap_add_view_plan(B, mo, o.kappa, F.stamp, cam6, &k, &phys);
        // label evidence (objprob.cpp:333-340): weight w = k / kappa_ref; the job adds
        // w max(log p, -60) to L_frag, from zeros when the object had none
        const bool txt = B.text_on && B.txt.dim == B.D;
        const double w = k / smax(1e-6, P.kappa_ref);
        if (s_job[a] >= 0) {
          UpdJob& j = B.upd_job[jbase + s_job[a]];
          j.k = k;
          j.phys = phys;
          j.w = txt ? w : 0.0;
          j.lzero = txt && !mo.has_lfrag;
          j.ltext = txt;
        }
        if (txt) {
          mo.lw_frag += w;
          mo.has_lfrag = 1;
        }
      }
      if (act == 1) {
          ++mo.n_ap_obs;
          if (o.wall_like) ++mo.n_wall_obs;
          if (o.struct_look) ++mo.n_struct_look;
          mo.wall_like = 2 * mo.n_wall_obs >= mo.n_ap_obs;
          if (!o.sec) {
            const double dt_seen = F.stamp - mo.last_seen;
            if (mo.parent && dist3(mo.pos, o.pos) > 0.3) mo.parent = 0;
            if (mo.last_kf != F.stamp) ++mo.n_obs;
            mo.last_kf = F.stamp;
            mo.rename = B.text_on;   // seen this keyframe (objmap.cpp:1007-1008)
            const int kd = kind_of(B, mo.cls);
            const bool big = kd == KIND_STATIC || kd == KIND_STRUCT_OBJ ||
                             smax(smax(mo.hi[0] - mo.lo[0], mo.hi[1] - mo.lo[1]), smax(o.ext[0], o.ext[1])) > P.big;
            bool snap = false;
            if (P.move_n > 0 && mo.trk_t > 0 && mo.held_by < 0 && !o.trunc && F.cam_steady) {
              const double dt = F.stamp - mo.trk_t;
              const double sx = o.pos[0] - mo.trk_pos[0], sy = o.pos[1] - mo.trk_pos[1];
              const double sp = dt > 1e-6 && dt <= 0.6 ? sqrt(sx * sx + sy * sy) / dt : 0.0;
              const bool same_dir = sx * mo.trk_step[0] + sy * mo.trk_step[1] > 0;
              mo.mv_cnt = sp > P.move_v && (same_dir || mo.mv_cnt == 0) ? mo.mv_cnt + 1 : 0;
              mo.trk_step[0] = sx;
              mo.trk_step[1] = sy;
              const double rx = o.pos[0] - mo.pos[0], ry = o.pos[1] - mo.pos[1];
              const double away = sqrt(rx * rx + ry * ry);
              const bool moving = F.stamp - mo.moving_t < 1.0;
              const bool left = away > smax(P.move_min_d, 0.5 * smax(o.ext[0], o.ext[1])) &&
                                box_overlap(o.lo, o.hi, mo.lo, mo.hi, P.merge_min_ext) < 0.1;
              if (mo.mv_cnt >= P.move_n && (moving || left)) {
                if (!moving) mo.move_from_t = F.stamp;
                mo.moving_t = F.stamp;
                snap = true;
              } else if (moving && sp > 0.5 * P.move_v) {
                snap = true;
                mo.moving_t = F.stamp;
              }
            }
            if (!o.trunc) {
              for (int k = 0; k < 3; ++k) mo.trk_pos[k] = o.pos[k];
              mo.trk_t = F.stamp;
            }
            if (snap) {
              double d3[3];
              for (int k = 0; k < 3; ++k) {
                d3[k] = o.pos[k] - mo.pos[k];
                mo.pos[k] = o.pos[k]; mo.ext[k] = o.ext[k]; mo.lo[k] = o.lo[k]; mo.hi[k] = o.hi[k];
              }
              CloudRec& C = B.clouds[cslot_glob(B, m, mo)];
              if (C.n > 0 && !(d3[0] == 0 && d3[1] == 0 && d3[2] == 0)) {   // ObjCloud::translate (cloud.cpp:79-84)
                for (int k = 0; k < 3; ++k) C.org[k] += d3[k];
                ++C.version;
                C.stamp = F.stamp;
              }
              if (dist3(mo.pos, mo.first_pos) > P.moved_d) mo.moved = 1;
              if (mo.moved && mo.state == 0) mo.state = 2;
              mo.parent = 0;
            }
            const bool fresh = mo.first_seen == F.stamp;
            for (int k = 0; k < 3 && !snap; ++k) {
              if (fresh) {
                mo.lo[k] = smin(mo.lo[k], o.lo[k]);
                mo.hi[k] = smax(mo.hi[k], o.hi[k]);
                mo.pos[k] = 0.5 * (mo.lo[k] + mo.hi[k]);
                mo.ext[k] = mo.hi[k] - mo.lo[k];
                continue;
              }
              if (big) {
                const double lo = smax(smin(mo.lo[k], o.lo[k]), mo.lo[k] - P.grow_max);
                const double hi = smin(smax(mo.hi[k], o.hi[k]), mo.hi[k] + P.grow_max);
                if (hi - lo <= P.max_ext) { mo.lo[k] = lo; mo.hi[k] = hi; }
                mo.pos[k] = 0.5 * (mo.lo[k] + mo.hi[k]);
                mo.ext[k] = mo.hi[k] - mo.lo[k];
              } else {
                const double K = kalman_gain(mo.P[k], P.ap_q_pos, dt_seen, kalman_R(P.ap_r0, P.ap_r1, o.zmed, o.trunc, o.ext[k]));
                mo.pos[k] += K * (o.pos[k] - mo.pos[k]);
                mo.lo[k] += K * (o.lo[k] - mo.lo[k]);
                mo.hi[k] += K * (o.hi[k] - mo.hi[k]);
                mo.ext[k] = mo.hi[k] - mo.lo[k];
              }
              if (big) kalman_big(mo.P[k], P.ap_q_pos, dt_seen, P.ap_r0 + P.ap_r1 * o.zmed, mo.ext[k]);
            }
            mo.score = (mo.score < o.score) ? o.score : mo.score;
            mo.max_det_z = smax(mo.max_det_z, o.zmed);
            mo.last_seen = F.stamp;
            mo.misses = 0;
            if (mo.state == 1) {
              mo.state = mo.moved ? 2 : 0;
              s_evf[a] |= 1;   // state event, numbered in P3
            }
            if (!mo.confirmed && (int)mo.n_obs >= P.confirm) {
              mo.confirmed = 1;
              s_evf[a] |= 2;   // confirmation event, numbered in P3
            }
          }
      }
    }
  }
  __syncthreads();
  // P3: events in observation order (new object: 0; update: state change 6, confirmation 1)
  if (tid == 0) {
    for (int a = 0; a < nobs; ++a) {
      const int act = s_act[a];
      if (!act) continue;
      const ObjRec& mo = REC[obs_rec[a]];
      if (act == 2) {
        push_event_l(B, m, F.stamp, mo, 0, (2u << 24) | (uint32_t)evn++, ev_base, &evl);
      } else {
        if (s_evf[a] & 1) push_event_l(B, m, F.stamp, mo, 6, (2u << 24) | (uint32_t)evn++, ev_base, &evl);
        if (s_evf[a] & 2) push_event_l(B, m, F.stamp, mo, 1, (2u << 24) | (uint32_t)evn++, ev_base, &evl);
      }
    }
    R->next_id = next_id;
    R->n_obj = n_obj;
    R->n_free = n_free;
    R->n_cfree = n_cfree;
    R->n_events = ev_base + evl;
    R->st.n_bridge += n_book[0];
    R->st.n_assoc += n_book[1];
    R->st.n_blocked += n_book[2];
    R->st.n_new += n_new;
    R->n_evn = evn;
    B.upd_n[2 * m] = njobs;
    B.upd_n[2 * m + 1] = ntg;
  }
  __syncthreads();
  // write back every staged record and the job targets
  for (int r = tid >> 5; r < nobs; r += blockDim.x >> 5)
    if (rec_slot[r] >= 0) rec_load(&B.objs[oglob(B, m, rec_slot[r])], &REC[r]);
  for (int c = tid; c < ntg; c += blockDim.x) B.upd_tg[(size_t)m * B.max_det + c] = tg_og[c];
}

// The D-length part of apAddView for every target object of the frame: one CTA per object
// applies that object's jobs in observation order (r_frag += float(k z), the fp16 view copy),
// then |r_frag|^2 and mu (objprob.cpp:228-240).  Objects are independent, so they run in
// parallel; each thread owns the same elements across jobs, so the jobs need no barrier.
__global__ void __launch_bounds__(UPD_THREADS) k_update_vec(Batch B) {
  __shared__ BlockScratch bs;
  const int c = blockIdx.x, m = B.map0 + blockIdx.y, tid = threadIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active || c >= B.upd_n[2 * m + 1]) return;
  const size_t base = (size_t)m * B.max_det;
  const size_t og = (size_t)B.upd_tg[base + c];
  const int nj = B.upd_n[2 * m];
  float* r = B.rfrag + og * B.D;
  int nmine = 0;
  for (int jj = 0; jj < nj; ++jj) {
    const UpdJob j = B.upd_job[base + jj];
    if (j.tg != c) continue;
    ++nmine;
    uint16_t* vz = B.views + (og * (B.topk + 1) + j.phys) * B.D;
    for (int i = tid; i < B.D; i += blockDim.x) {
      const float zi = emb_at(F.emb, F.emb_dtype, B.D, j.det, i);
      r[i] = (j.zero ? 0.f : r[i]) + (float)(j.k * (double)zi);
      vz[i] = ref_f2h(zi);
    }
    if (j.ltext) {   // L_frag += w max(log p, -60) (objprob.cpp:335-339: float per label)
      const int C = B.txt.n_labels;
      float* L = B.lfrag + og * C;
      const float* ll = B.llz + ((size_t)m * B.max_det + j.det) * C;
      for (int l = tid; l < C; l += blockDim.x) L[l] = (j.lzero ? 0.f : L[l]) + (float)(j.w * smax((double)ll[l], -60.0));
    }
  }
  if (tid == 0) wk_add(&B.maps[m], SMG_WK_UPD, nmine);
  __syncthreads();
  refresh_nrm(B, og, bs);
}
