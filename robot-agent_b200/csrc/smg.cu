// C ABI of the B200 scenemap objprob update (include/smg.h): parameters, batch allocation,
// the per-keyframe launch chain, and device->host getters.
//
// Launch chain of one smg_push_frames call (all maps of the batch in every launch):
//   k_begin         per-frame resets
//   k_hands         grasp / hold / release, support links (objmap.cpp:435-506; only once a
//                   gripper of the batch has closed)
//   k_merge_pairs   apMergePass pair evaluation        (objmap.cpp:1154-1200)
//   k_merge_apply   greedy merges (absorb + apMerge)   (objmap.cpp:1202-1224)
//   k_obs           back-projection .. plane fit       (objmap.cpp:645-765)
//   k_obs_finalize  structural decisions, obs list     (objmap.cpp:576-621)
//   k_assoc         association                        (objmap.cpp:767-810)
//   k_update        fusion, update, new objects        (objmap.cpp:811-997)
//   k_absent        absence / misses                   (objmap.cpp:1020-1061)
//   k_relink        cloud lists + relink               (objmap.cpp:1010-1019, 1062)
//   k_struct        merged-cloud geometry              (objmap.cpp:1064, 1255-1319)
//   k_prune         drop / prune, cloud targets        (objmap.cpp:1066-1073)
//   k_markview      seen cells                         (objmap.cpp:1084)
//   k_cloud_add     ObjectMap::addPoints + contact     (capi.cpp:986-992, cloud.cpp:86-127)
//   k_grid          makeScan + insert policy + insert  (mapper2d.cpp:27-87)
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "k_grid.cuh"
#include "k_occ.cuh"
#include "k_gemm_assoc.cuh"
#include "k_text.cuh"
#include "k_gather.cuh"
#include "k_reenc.cuh"
#include "k_hands.cuh"
#include "k_views.cuh"
#include "k_textmap.cuh"
#include "k_walls.cuh"
#include "k_snap.cuh"

#include <cudaTypedefs.h>

#define PF_THREADS 256   // CTA size of the batched plane fit (the block sums' tree follows it)

static thread_local std::string g_err;
static int fail(int code, const char* msg) {
  g_err = msg;
  return code;
}
#define CK(x)                                                     \
  do {                                                            \
    cudaError_t e_ = (x);                                         \
    if (e_ != cudaSuccess) {                                      \
      g_err = std::string(#x) + ": " + cudaGetErrorString(e_);    \
      return SMG_ERR_DEVICE;                                      \
    }                                                             \
  } while (0)

struct smg_batch {
  Batch B;
  int dev;
  int max_w, max_h;
  std::vector<void*> allocs;
  static const int kRing = 4;
  FrameDev* h_ring = nullptr;     // pinned, kRing x M descriptors
  cudaEvent_t ring_ev[4] = {nullptr, nullptr, nullptr, nullptr};
  bool ring_used[4] = {false, false, false, false};
  long long n_push = 0;
  FrameDev* h_frames = nullptr;   // current ring slot
  // stream groups: the maps are split into `groups` ranges, each with its own chain stream (the
  // caller's for group 0) and occupancy side stream; host inputs arrive on s_copy
  static constexpr int kGroupsMax = 8;
  int groups = 1;
  bool host_gather = getenv("SMG_HOST_GATHER") == nullptr || atoi(getenv("SMG_HOST_GATHER")) != 0;
  cudaStream_t s_grp[kGroupsMax] = {}, s_gridg[kGroupsMax] = {}, s_copy = nullptr, s_dma = nullptr;
  cudaEvent_t ev_wall[kGroupsMax] = {};   // a group's wall extraction (grid stream) is done
  cudaEvent_t ev_fork[kGroupsMax] = {}, ev_join[kGroupsMax] = {}, ev_copied[kGroupsMax] = {}, ev_gdone[kGroupsMax] = {},
              ev_dma[kGroupsMax] = {};
  cudaEvent_t ev_up = nullptr, ev_done = nullptr;
  bool dbg_sync = getenv("SMG_DEBUG_SYNC") != nullptr;   // synchronise + check after every launch
  long long dbg_last = 0;
  float* d_depth = nullptr;       // staging for SMG_MEM_HOST
  uint16_t* d_label = nullptr;
  unsigned char* d_emb = nullptr;
  uint16_t* d_depth_mm = nullptr;  // staging of host millimetre depth
  uint32_t* d_mask = nullptr;      // staging of host detector bit masks: M x max_det x mask_words_max
  uint8_t* d_rgba = nullptr;       // staging of host RGBA images (allocated on first use)
  // wall segments of host frames (allocated by the first push that carries some): a pinned
  // ring (kRing x M x SMG_WALL_SEGS_MAX x 4, slot = the descriptor ring's) and two device
  // staging sets, packed frame after frame
  double* h_wall = nullptr;
  double* d_wall = nullptr;
  float* d_wstate = nullptr;   // smg_wall_state's result
  // smg_snapshot scratch (allocated on the first call; the point records grow as needed)
  smg_snap_object* d_snap_rec = nullptr;
  smg_snap_object* d_snap_out = nullptr;
  int32_t* d_snap_cnt = nullptr;
  int32_t* d_snap_src = nullptr;
  int32_t* d_snap_moff = nullptr;
  int64_t* d_snap_npts = nullptr;
  int64_t* d_snap_poff = nullptr;
  uint8_t* d_snap_pts = nullptr;
  size_t snap_pts_cap = 0;
  // The staging above is double-buffered: push k fills set k % 2 while the chain of push k - 1
  // still reads the other set, so a push's host-to-device copies overlap the previous chain.
  // ev_set[s] marks the end of the last chain that read set s.
  int stage_set = 0;
  cudaEvent_t ev_set[2] = {nullptr, nullptr};
  FrameDev* frames_base = nullptr;   // device descriptors: set s at frames_base + s * M
  // asynchronous association reads (smg_get_assoc_all_async): a ring of device buffers + events
  static const int kReads = 4;
  uint32_t* d_aids = nullptr;        // kReads x M x max_det
  cudaEvent_t ev_rd[4] = {nullptr, nullptr, nullptr, nullptr};
  long long n_reads = 0;
  bool views_alloc = false;        // best-view records and image slots allocated
  bool views_push = false;         // some map of the current push picks views
  // whole-view answers (smg_set_object_embeddings): staging of up to M * RE_CAND entries, and the
  // stamp of every map's last keyframe (the stamp the reference gives the whole views)
  int32_t* d_wv_map = nullptr;
  uint32_t* d_wv_id = nullptr;
  float* d_wv_emb = nullptr;
  double* d_wv_stamp = nullptr;
  std::vector<double> last_stamp;
  size_t mask_words_max = 0;       // ceil(max_w * max_h / 32)
  std::vector<double> last_cam_t, last_cam_fwd;
  // updateHands' per-hand gripper state of every map (ObjectMap::closed_, gref_, gref_t_, tried_;
  // objmap.hpp:320-323), [2 * m + h]
  std::vector<int> h_closed, h_tried;
  std::vector<double> h_gref, h_gref_t;
  bool hands_on = false;   // some map has tried a grasp: held objects and support links may exist
  long long launches = 0;
  long long h2d_host = 0;   // host-input bytes copied by the copy engines
  cudaStream_t last_stream = nullptr;
  // per-kernel event timing
  bool timing = false;
  std::vector<cudaEvent_t> ev_pool;
  std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> ev_used;
  double k_ms[SMG_NUM_KERNELS] = {0};
  long long k_n[SMG_NUM_KERNELS] = {0};
};

static const char* k_names[SMG_NUM_KERNELS] = {"k_begin", "k_merge_pairs", "k_merge_apply", "k_obs", "k_obs_finalize", "k_assoc",
                                               "k_update", "k_absent", "k_relink", "k_struct", "k_prune", "k_markview",
                                               "k_cloud_add", "k_grid", "k_reenc", "k_hands", "k_views", "k_walls"};

static cudaEvent_t ev_get(smg_batch* b) {
  if (b->ev_pool.empty()) {
    cudaEvent_t e;
    cudaEventCreate(&e);
    return e;
  }
  cudaEvent_t e = b->ev_pool.back();
  b->ev_pool.pop_back();
  return e;
}

extern "C" int smg_destroy(smg_batch* b);
template <class T>
static int dalloc(smg_batch* b, T** p, size_t n, int fill_byte = 0) {
  void* q = nullptr;
  const size_t bytes = std::max<size_t>(n, 1) * sizeof(T);
  CK(cudaMalloc(&q, bytes));
  CK(cudaMemset(q, fill_byte, bytes));
  b->allocs.push_back(q);
  *p = (T*)q;
  return SMG_OK;
}
#define DA(ptr, n)                                 \
  do {                                             \
    int r_ = dalloc(b, &(ptr), (size_t)(n));       \
    if (r_) { smg_destroy(b); return r_; }         \
  } while (0)

__global__ void k_fill_d(double* p, size_t n, double v) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) p[i] = v;
}
__global__ void k_fill_i64(int64_t* p, size_t n, int64_t v) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) p[i] = v;
}
__global__ void k_fill_i8(int8_t* p, size_t n, int8_t v) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) p[i] = v;
}


extern "C" {

const char* smg_last_error(void) { return g_err.c_str(); }

int smg_params_size(void) { return (int)sizeof(smg_params); }

int smg_params_set_cloud(smg_params* p, double voxel, int cap) {
  if (!p) return SMG_ERR_ARGS;
  if (voxel > 0) p->voxel = voxel;
  if (cap > 0) p->cloud_cap = cap;
  return SMG_OK;
}

int smg_params_default(smg_params* p) {
  if (!p) return SMG_ERR_ARGS;
  memset(p, 0, sizeof(*p));
  // ObjParams (objmap.hpp:50-129)
  p->min_points = 20;
  p->zmin = 0.15f; p->zmax = 3.0f; p->hand_r = 0.10f; p->hand_frac = 0.5f;
  p->big = 0.5; p->confirm = 2; p->prune_s = 10.0; p->moved_d = 0.15; p->gone_misses = 3; p->gone_min_s = 2.0;
  p->mad_k = 3.0; p->mad_floor = 0.10; p->grow_max = 0.25; p->max_ext = 4.0; p->occl = 0.10; p->min_px = 6;
  p->self_pad = 0.01; p->step = 1; p->max_pts = 6000; p->voxel = 0.02; p->cloud_cap = 8000; p->cloud_hand_r = 0.05;
  p->body_r = 0.22; p->merge_min_ext = 0.05; p->floor_h = 0.05; p->absent_samples = 48; p->absent_vis = 0.5;
  p->absent_min_px = 12; p->absent_det_k = 1.15; p->gone_misses_big = 6; p->gone_min_s_big = 4.0; p->spurious_obs = 5;
  p->gone_view_d = 0.5; p->gone_step_d = 0.10; p->gone_step_deg = 5.0; p->gone_eps = 0.02;
  p->link_v = 1.0; p->link_d0 = 1.0; p->link_max_d = 8.0; p->link_min_obs = 3; p->link_wait_s = 30.0;
  p->link_window_s = 180.0; p->link_view_gap_s = 5.0; p->view_cell = 0.5;
  p->move_n = 3; p->move_v = 0.3; p->move_min_d = 0.25; p->move_max_cam_w = 0.6;
  p->ap_q_pos = 1e-4; p->ap_r0 = 0.02; p->ap_r1 = 0.01;
  // ApParams (objprob.hpp:56-142)
  p->same_p = 0.6; p->merge_p = 0.7;
  const double w[8] = {-5.116, 4.553, -4.976, 0.376, 8.814, 1.824, -0.186, 0.0};
  const double wm[8] = {-4.265, 1.094, -3.378, 0.627, 8.823, 3.205, -2.500, 1.717};
  memcpy(p->w, w, sizeof w);
  memcpy(p->wm, wm, sizeof wm);
  p->guard_obj = 0.6; p->guard_obs = 0.2; p->name_veto = 0; p->bridge_drop = 0; p->frame_group = 1;
  p->cos0 = 0.75; p->gate = 0.30; p->contact_cell = 0.04; p->contact_samples = 160; p->topk = 5;
  p->temper_d = 0.30; p->temper_deg = 15.0; p->temper = 0.3; p->kappa_ref = 3000;
  p->plane_thick = 0.035; p->ransac_tau0 = 0.01; p->ransac_tau_k = 0.0025; p->ransac_tau_max = 0.05; p->obj_tau = 0.02;
  p->plane_inl = 0.8; p->obj_plane_inl = 0.92; p->ransac_iters = 64;
  p->wall_vert = 0.30; p->ceil_z = 2.0; p->horiz = 0.85; p->floor_z = 0.06; p->ceil_band = 0.35; p->ceil_frac = 0.5;
  p->ceil_wide = 0.6; p->tall_h = 1.7; p->tall_floor = 0.3; p->tall_ceil = 0.4; p->tall_w = 1.5; p->tall_ps = 0.3;
  p->tall_w_any = 3.0; p->obj_wall_span = 1.5; p->obj_wall_top = 1.9; p->obj_wall_h = 1.0; p->obj_thick = 0.04;
  p->struct_obj_p = 0.6; p->struct_obj_min_views = 2; p->link_cos = 0.8;
  // KappaParams (bestview.hpp:67-69)
  p->kap_k0 = 4369; p->kap_s0 = 40; p->kap_trunc = 1.0; p->kap_d0 = 100.0; p->kap_occ = 1.0; p->kap_blur_w = 0.0;
  // GridParams (grid.hpp:18-21), ScanParams (scan.hpp:37-48), MapperParams (mapper2d.hpp:14-26)
  p->grid_res = 0.05f; p->l_hit = 0.85f; p->l_miss = -0.4f; p->l_min = -4.f; p->l_max = 4.f;
  p->scan_zmin = 0.3f; p->scan_zmax = 3.0f; p->band_lo = 0.05f; p->band_hi = 0.50f; p->bins = 720;
  p->self_r = 0.22f; p->eef_r = 0.08f; p->arm_r = 0.06f;
  for (int s = 0; s < 2; ++s) { p->shoulder[s][0] = -0.05f; p->shoulder[s][1] = 0.f; p->shoulder[s][2] = 0.25f; }
  p->match_hi = 3.0f; p->vert_nz = 0.7f; p->match_cell = 0.025f; p->dense = 1;
  p->change_bins = 2; p->change_cells = 1; p->still_every = 50;
  p->reenc_max = 8; p->reenc_gain = 1.3; p->reenc_min_vis = 0.5; p->reenc_min_px = 24;   // objprob.hpp:90-93
  // hands (objmap.hpp:66-76)
  p->grasp_r = 0.12; p->grip_closed = 0.6f; p->n_hands = 1;
  p->grasp_max_w = 0.06; p->grasp_min_gap = 0.005; p->grasp_w_tol = 0.025; p->grip_settle_s = 0.2; p->grip_settle_eps = 0.01;
  const double gg[7][2] = {{0.0, 0.0}, {0.095, 0.01}, {0.231, 0.02}, {0.347, 0.03}, {0.408, 0.04}, {0.5236, 0.0551}, {0.7854, 0.0933}};
  p->n_grip_gap = 7;
  memcpy(p->grip_gap, gg, sizeof gg);
  // text-model rules (objprob.hpp:84-136)
  p->name_tau = 0.5; p->name_wmax = 6.0; p->size_w = 1.0; p->whole_w = 1.0; p->geo_w = 3.0; p->flat_max_w = 2.2;
  p->wall_big = 1.0; p->struct_p = 0.5;
  p->wall_d = 0.12; p->wall_frac = 0.6; p->through_d = 0.20; p->bridge_max = 0.0;
  p->obj_flat_thick = 0.012; p->obj_flat_d = 0.10; p->obj_flat_frac = 0.7; p->flat_keep_p = 0.5;
  p->so_dw_w = 2.2; p->so_dw_thick = 0.45; p->so_max_h = 2.8; p->so_pillar = 1.0; p->so_stairs = 6.0; p->so_dw_min = 0.3;
  p->so_hide_k = 1.5; p->wallhug_frac = 0.75; p->wallhug_w = 2.0; p->big_vinl = 0.5;
  p->struct_look_block = 1; p->so_min_obs = 12;
  return SMG_OK;
}

// ObjectMap::applyParams key table (scenemap src/objmap.cpp:135-180).  Keys whose feature the
// device path does not run (the inspect pass, the export filter) only ever take
// the reference default here: any other value is reported as unsupported, so a parameter file
// cannot change the reference's behaviour and leave this one unchanged without an error.
int smg_params_apply(smg_params* p, const char* kv) {
  if (!p) return SMG_ERR_ARGS;
  if (!kv || !*kv) return 0;
  // d/i: the field the key sets; dflt: for keys of features this build does not run (d == i ==
  // null), the reference default (objprob.hpp:84-136, inspect.hpp:19), the only value accepted
  struct K { const char* n; double* d; int32_t* i; double dflt; };
  const K keys[] = {
      {"floor_h", &p->floor_h, 0, 0}, {"absent_samples", 0, &p->absent_samples, 0}, {"absent_vis", &p->absent_vis, 0, 0},
      {"absent_min_px", &p->absent_min_px, 0, 0}, {"absent_det_k", &p->absent_det_k, 0, 0}, {"gone_misses", 0, &p->gone_misses, 0},
      {"gone_min_s", &p->gone_min_s, 0, 0}, {"gone_misses_big", 0, &p->gone_misses_big, 0}, {"gone_min_s_big", &p->gone_min_s_big, 0, 0},
      {"gone_view_d", &p->gone_view_d, 0, 0}, {"gone_eps", &p->gone_eps, 0, 0}, {"gone_step_d", &p->gone_step_d, 0, 0},
      {"gone_step_deg", &p->gone_step_deg, 0, 0}, {"spurious_obs", 0, &p->spurious_obs, 0}, {"link_v", &p->link_v, 0, 0},
      {"link_d0", &p->link_d0, 0, 0}, {"link_max_d", &p->link_max_d, 0, 0}, {"link_min_obs", 0, &p->link_min_obs, 0},
      {"link_wait_s", &p->link_wait_s, 0, 0}, {"link_window_s", &p->link_window_s, 0, 0}, {"link_view_gap_s", &p->link_view_gap_s, 0, 0},
      {"view_cell", &p->view_cell, 0, 0}, {"confirm", 0, &p->confirm, 0}, {"move_v", &p->move_v, 0, 0}, {"move_n", 0, &p->move_n, 0},
      {"move_min_d", &p->move_min_d, 0, 0}, {"move_max_cam_w", &p->move_max_cam_w, 0, 0}, {"self_pad", &p->self_pad, 0, 0},
      {"inspect", 0, 0, 0},
      {"ap_same_p", &p->same_p, 0, 0}, {"ap_merge_p", &p->merge_p, 0, 0}, {"ap_gate", &p->gate, 0, 0}, {"ap_name_tau", &p->name_tau, 0, 0},
      {"ap_name_wmax", &p->name_wmax, 0, 0}, {"ap_size_w", &p->size_w, 0, 0}, {"ap_kappa_ref", &p->kappa_ref, 0, 0}, {"ap_temper", &p->temper, 0, 0},
      {"ap_wall_big", &p->wall_big, 0, 0}, {"ap_struct_p", &p->struct_p, 0, 0}, {"ap_ceil_z", &p->ceil_z, 0, 0}, {"ap_struct_obj_p", &p->struct_obj_p, 0, 0},
      {"ap_obj_wall_span", &p->obj_wall_span, 0, 0}, {"ap_obj_wall_top", &p->obj_wall_top, 0, 0}, {"ap_reenc_max", 0, &p->reenc_max, 0},
      {"ap_reenc_gain", &p->reenc_gain, 0, 0}, {"ap_link_cos", &p->link_cos, 0, 0}, {"ap_whole_w", &p->whole_w, 0, 0},
      {"ap_export_named", 0, 0, 1}, {"ap_guard_obj", &p->guard_obj, 0, 0}, {"ap_guard_obs", &p->guard_obs, 0, 0},
      {"ap_geo_w", &p->geo_w, 0, 0}, {"ap_name_veto", &p->name_veto, 0, 0}, {"ap_through_d", &p->through_d, 0, 0}, {"ap_bridge_max", &p->bridge_max, 0, 0},
      {"ap_frame_group", 0, &p->frame_group, 0}, {"ap_struct_obj_min_views", 0, &p->struct_obj_min_views, 0},
      {"ap_plane_inl", &p->plane_inl, 0, 0}, {"ap_obj_plane_inl", &p->obj_plane_inl, 0, 0}, {"ap_ransac_tau0", &p->ransac_tau0, 0, 0},
      {"ap_ransac_tau_k", &p->ransac_tau_k, 0, 0}, {"ap_obj_tau", &p->obj_tau, 0, 0}, {"ap_ransac_iters", 0, &p->ransac_iters, 0},
      {"ap_so_dw_w", &p->so_dw_w, 0, 0}, {"ap_so_dw_thick", &p->so_dw_thick, 0, 0}, {"ap_so_max_h", &p->so_max_h, 0, 0}, {"ap_so_pillar", &p->so_pillar, 0, 0},
      {"ap_so_stairs", &p->so_stairs, 0, 0}, {"ap_wallhug_frac", &p->wallhug_frac, 0, 0}, {"ap_wallhug_w", &p->wallhug_w, 0, 0},
      {"ap_struct_look_block", 0, &p->struct_look_block, 0}, {"ap_flat_max_w", &p->flat_max_w, 0, 0}, {"ap_tall_h", &p->tall_h, 0, 0}, {"ap_tall_w", &p->tall_w, 0, 0},
      {"ap_tall_ps", &p->tall_ps, 0, 0}, {"ap_tall_w_any", &p->tall_w_any, 0, 0}, {"ap_big_vinl", &p->big_vinl, 0, 0}, {"ap_so_dw_min", &p->so_dw_min, 0, 0},
      {"ap_so_hide_k", &p->so_hide_k, 0, 0},
      {"ap_w0", &p->w[0], 0, 0}, {"ap_w1", &p->w[1], 0, 0}, {"ap_w2", &p->w[2], 0, 0}, {"ap_w3", &p->w[3], 0, 0}, {"ap_w4", &p->w[4], 0, 0},
      {"ap_w5", &p->w[5], 0, 0}, {"ap_w6", &p->w[6], 0, 0}, {"ap_w7", &p->w[7], 0, 0},
      {"ap_wm0", &p->wm[0], 0, 0}, {"ap_wm1", &p->wm[1], 0, 0}, {"ap_wm2", &p->wm[2], 0, 0}, {"ap_wm3", &p->wm[3], 0, 0},
      {"ap_wm4", &p->wm[4], 0, 0}, {"ap_wm5", &p->wm[5], 0, 0}, {"ap_wm6", &p->wm[6], 0, 0}, {"ap_wm7", &p->wm[7], 0, 0},
      {"ap_cos0", &p->cos0, 0, 0}, {"ap_bridge_drop", 0, &p->bridge_drop, 0},
      {"kap_k0", &p->kap_k0, 0, 0}, {"kap_s0", &p->kap_s0, 0, 0}, {"kap_trunc", &p->kap_trunc, 0, 0}, {"kap_d0", &p->kap_d0, 0, 0}};
  // boolean keys (bool fields in the reference: v != 0)
  auto is_bool = [](const char* n) {
    return !strcmp(n, "ap_frame_group") || !strcmp(n, "ap_bridge_drop") || !strcmp(n, "inspect") || !strcmp(n, "ap_export_named") ||
           !strcmp(n, "ap_struct_look_block");
  };
  int n_bad = 0;
  std::string unsupported;
  std::string s(kv);
  size_t a = 0;
  while (a < s.size()) {
    size_t b = s.find(',', a);
    if (b == std::string::npos) b = s.size();
    const std::string item = s.substr(a, b - a);
    a = b + 1;
    const size_t q = item.find('=');
    if (q == std::string::npos) continue;
    const std::string k = item.substr(0, q);
    const double v = atof(item.c_str() + q + 1);
    bool ok = false;
    for (const K& x : keys)
      if (k == x.n) {
        ok = true;
        if (x.d) *x.d = v;
        else if (x.i) *x.i = is_bool(x.n) ? (v != 0) : (int32_t)v;
        else if (is_bool(x.n) ? ((v != 0) != (x.dflt != 0)) : v != x.dflt)
          unsupported += (unsupported.empty() ? "" : ",") + k;
      }
    if (!ok) ++n_bad;
  }
  if (n_bad) {
    g_err = "unknown parameter key";
    return n_bad;
  }
  if (!unsupported.empty()) {
    g_err = "parameter keys of features this build does not run, set away from the reference default: " + unsupported;
    return SMG_ERR_UNSUPPORTED;
  }
  return 0;
}

int smg_destroy(smg_batch* b) {
  if (!b) return SMG_ERR_ARGS;
  for (auto& u : b->ev_used) { cudaEventDestroy(u.second.first); cudaEventDestroy(u.second.second); }
  for (auto e : b->ev_pool) cudaEventDestroy(e);
  for (void* p : b->allocs) cudaFree(p);
  if (b->h_ring) cudaFreeHost(b->h_ring);
  if (b->h_wall) cudaFreeHost(b->h_wall);
  if (b->d_snap_pts) cudaFree(b->d_snap_pts);
  for (auto e : b->ring_ev) if (e) cudaEventDestroy(e);
  for (int g = 0; g < smg_batch::kGroupsMax; ++g) {
    for (cudaEvent_t e : {b->ev_fork[g], b->ev_join[g], b->ev_copied[g], b->ev_gdone[g], b->ev_dma[g], b->ev_wall[g]}) if (e) cudaEventDestroy(e);
    for (cudaStream_t q : {b->s_grp[g], b->s_gridg[g]}) if (q) cudaStreamDestroy(q);
  }
  for (cudaEvent_t e : {b->ev_up, b->ev_done, b->ev_set[0], b->ev_set[1], b->ev_rd[0], b->ev_rd[1], b->ev_rd[2], b->ev_rd[3]})
    if (e) cudaEventDestroy(e);
  if (b->s_copy) cudaStreamDestroy(b->s_copy);
  if (b->s_dma) cudaStreamDestroy(b->s_dma);
  delete b;
  return SMG_OK;
}

// RANSAC adaptive-iteration table (host libm, like the reference): need = max(8,
// ceil(log(0.01) / log(1 - w^3))) for w = cnt / nsamp; 0 where the reference does not update it.
static const std::vector<int32_t>& need_table() {
  static const std::vector<int32_t> tab = [] {
    std::vector<int32_t> need((size_t)NEED_N * NEED_N, 0);
    for (int ns = 1; ns < NEED_N; ++ns)
      for (int c = 0; c <= ns; ++c) {
        const double w = double(c) / double(ns), pw = w * w * w;
        need[(size_t)ns * NEED_N + c] = pw > 1e-9 && pw <= 0.999999 ? std::max(8, int(std::ceil(std::log(0.01) / std::log(1.0 - pw)))) : 0;
      }
    return need;
  }();
  return tab;
}

static int pow2_at_least(long long n) {
  int v = 1;
  while (v < n) v <<= 1;
  return v;
}

int smg_create(const smg_params* p, int n_maps, int max_objects, int emb_dim, int max_w, int max_h, int max_det, int grid_w,
               int grid_h, int grid_x0, int grid_y0, int dev, smg_batch** out) {
  return smg_create_pooled(p, n_maps, max_objects, max_objects, emb_dim, max_w, max_h, max_det, grid_w, grid_h, grid_x0, grid_y0,
                           dev, out);
}

int smg_create_pooled(const smg_params* p, int n_maps, int max_objects, int max_clouds, int emb_dim, int max_w, int max_h,
                      int max_det, int grid_w, int grid_h, int grid_x0, int grid_y0, int dev, smg_batch** out) {
  if (!p || !out || n_maps <= 0 || max_objects <= 0 || max_clouds <= 0 || max_clouds > max_objects || emb_dim <= 0 || emb_dim > 2048 || max_w <= 0 || max_h <= 0 || max_det <= 0 ||
      max_det > SMG_MAX_DET || grid_w <= 0 || grid_h <= 0 || p->topk <= 0 || p->topk > SMG_TOPK_MAX || p->bins <= 0 ||
      p->bins > SMG_BINS_MAX || max_objects > PRUNE_MAX || p->n_grip_gap < 0 || p->n_grip_gap > 8 || p->cloud_cap <= 0 || p->voxel <= 0 || p->ransac_iters > RANSAC_MAX ||
      (size_t)max_h * ((max_w + 31) / 32) * 4 + RE_ZMAX * 4 > 227 * 1024)   // re-encode mask held in shared memory
    return fail(SMG_ERR_ARGS, "smg_create: bad arguments");
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || dev < 0 || dev >= ndev) return fail(SMG_ERR_DEVICE, "smg_create: no CUDA device");
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess || prop.major < 10)
    return fail(SMG_ERR_DEVICE, "smg_create: needs an sm_100 device");
  if (cudaSetDevice(dev) != cudaSuccess) return fail(SMG_ERR_DEVICE, "smg_create: cudaSetDevice");
  smg_batch* b = new smg_batch();
  b->dev = dev;
  b->max_w = max_w;
  b->max_h = max_h;
  Batch& B = b->B;
  memset(&B, 0, sizeof(B));
  const int M = n_maps, O = max_objects, D = emb_dim;
  const int CP = max_clouds;
  B.M = M; B.O = O; B.C = CP; B.D = D; B.topk = p->topk; B.max_det = max_det; B.W = max_w; B.H = max_h; B.map0 = 0;
  B.reenc_on = 1;
  B.p = *p;
  B.cap = 2 * p->cloud_cap;
  B.HC = pow2_at_least(2LL * B.cap);
  B.HCC = pow2_at_least(2LL * p->cloud_cap);
  {   // box scan bound: max_pts + rows + cols + 1 (objmap.cpp:652), at least cloud_cap for merges
    const long long pm = std::max<long long>((long long)p->max_pts + max_w + max_h + 1, p->cloud_cap);
    B.pmax = pow2_at_least(pm);
  }
  B.work_n = std::max(B.cap, B.pmax);
  B.work_stride = ((size_t)B.work_n * (4 * 16 + 8 + 4 + 8 + 16 + 4) + 64 + 255) / 256 * 256;
  B.gw_grid = grid_w; B.gh_grid = grid_h; B.gx0 = grid_x0; B.gy0 = grid_y0;
  B.view_slots = 8192;
  {
    const int step = std::max(1, (int)lround(max_w / 160.0));
    B.scan_pmax = ((max_w + step - 1) / step) * ((max_h + step - 1) / step);
  }
  B.cos_temper = cos(p->temper_deg * M_PI / 180.0);
  B.cos_gone_step = cos(p->gone_step_deg * M_PI / 180.0);
  B.inv_vox = (float)(1.0 / std::max(1e-3, p->voxel));
  B.inv_vox_cloud = (float)(1.0 / p->voxel);
  B.q_hit = (int16_t)lround(p->l_hit * 256);
  B.q_miss = (int16_t)lround(p->l_miss * 256);
  B.q_min = (int16_t)lround(p->l_min * 256);
  B.q_max = (int16_t)lround(p->l_max * 256);
  B.lut_off = -B.q_min;
  const size_t MO = (size_t)M * O;
  DA(B.maps, M);
  DA(B.frames, 2 * (size_t)M);   // two descriptor sets, alternating with the staging sets
  b->frames_base = B.frames;
  DA(B.objs, MO);
  DA(B.order, MO);
  DA(B.freel, MO);
  const size_t MC = (size_t)M * CP;
  DA(B.cfreel, MC);
  DA(B.assoc, (size_t)M * max_det);
  DA(B.rfrag, MO * D);
  DA(B.mu, MO * D);
  DA(B.views, MO * (B.topk + 1) * D);
  DA(B.clouds, MC);
  DA(B.cpts, MC * B.cap);
  DA(B.crgb, MC * B.cap);
  DA(B.chkey, MC * B.HC);
  DA(B.chidx, MC * B.HC);
  DA(B.chgen, MC * B.HC);
  DA(B.cbits, MC * 2 * CB_WORDS);
  DA(B.ckey, MC * B.HCC);
  DA(B.cgen, MC * B.HCC);
  const size_t MD = (size_t)M * max_det;
  DA(B.px, MD * 4 * B.pmax);
  DA(B.ppix, MD * 2 * B.pmax);
  DA(B.pk, MD * 3 * B.pmax);
  DA(B.cxyz, MD * 3 * B.pmax);
  DA(B.cpx, MD * 2 * B.pmax);
  DA(B.sel, MD * 4 * B.pmax);
  DA(B.obs, MD);
  DA(B.obs_list, MD);
  DA(B.touched, MO + max_det);
  DA(B.obj_hit, MO + max_det);
  DA(B.ptsl, MD);
  DA(B.gdot, MD * max_det);
  DA(B.tgt_slot, MO);
  DA(B.events, (size_t)M * SMG_MAX_EVENTS);
  DA(B.mcand_p, MO * 8);
  DA(B.mcand_ab, MO * 8 * 2);
  DA(B.mcand_key, MO * 8);
  DA(B.mcand_n, M);
  DA(B.mgl, (size_t)M * MGL_CAP);
  DA(B.mgl_n, 2 * (size_t)M);
  B.re_words = (size_t)max_h * ((max_w + 31) >> 5);
  DA(B.reenc, (size_t)M * RE_CAND);
  DA(B.reenc_bits, (size_t)M * RE_CAND * B.re_words);
  DA(B.pcache, (size_t)M * PCACHE_SLOTS);
  DA(B.sscr, (size_t)M * STRUCT_CTAS * STRUCT_SCR);
  DA(B.upd_job, MD);
  DA(B.upd_tg, MD);
  DA(B.upd_n, (size_t)M * 2);
  DA(B.vkey, (size_t)M * B.view_slots);
  DA(B.vfirst, (size_t)M * B.view_slots * SMG_VIEW_BANDS);
  DA(B.need_tab, NEED_N * NEED_N);
  DA(B.wsegs, (size_t)M * SMG_WALL_SEGS_MAX * 4);
  const size_t G = (size_t)M * grid_w * grid_h;
  DA(B.gL, G);
  DA(B.gc8, G);
  DA(B.gflags, G);
  DA(B.gcold, G);
  DA(B.gcnt, G);
  DA(B.gtouch, G);
  CK(cudaMemset(B.gtouch, 0xff, sizeof(unsigned long long) * G));
  const int nlut = B.q_max - B.q_min + 1;
  DA(B.lut8, nlut);
  DA(B.lutp, nlut);
  DA(B.sP, (size_t)M * B.scan_pmax);
  DA(B.bin_cos, p->bins);
  DA(B.bin_sin, p->bins);
  DA(B.hit_key, (size_t)M * p->bins);
  DA(B.floor_r, (size_t)M * p->bins);
  DA(B.sig, (size_t)M * p->bins);
  DA(B.ins_sig, (size_t)M * p->bins);
  DA(B.mkey, (size_t)M * B.scan_pmax);
  DA(B.mval, (size_t)M * B.scan_pmax);
  DA(B.mh_key, (size_t)M * MH_SLOTS);
  DA(B.mh_first, (size_t)M * MH_SLOTS);
  DA(B.mh_cell, (size_t)M * MH_SLOTS);
  DA(B.mcell_first, (size_t)M * B.scan_pmax);
  DA(B.mcell_cnt, (size_t)M * B.scan_pmax);
  DA(B.mcell_off, (size_t)M * B.scan_pmax);
  DA(B.mcell_pix, (size_t)M * B.scan_pmax);
  DA(B.sc_pts, (size_t)M * (2 * SMG_BINS_MAX + SMG_MATCH_CELLS) * 4);
  DA(B.work, (size_t)M * WORK_SLOTS * B.work_stride);
  DA(b->d_depth, 2 * (size_t)M * max_w * max_h);
  DA(b->d_label, 2 * (size_t)M * max_w * max_h);
  DA(b->d_emb, 2 * (size_t)M * max_det * D * 4);
  DA(b->d_depth_mm, 2 * (size_t)M * max_w * max_h);
  DA(b->d_wv_map, (size_t)M * RE_CAND);
  DA(b->d_wv_id, (size_t)M * RE_CAND);
  DA(b->d_wv_emb, (size_t)M * RE_CAND * D);
  DA(b->d_wv_stamp, M);
  DA(B.rwhole, MO * D);
  b->last_stamp.assign(M, 0.0);
  b->mask_words_max = ((size_t)max_w * max_h + 31) / 32;
  DA(b->d_mask, 2 * (size_t)M * max_det * b->mask_words_max);
  // host-side initial state
  {
    std::vector<MapRec> maps((size_t)M);
    for (auto& r : maps) {
      memset(&r, 0, sizeof(r));
      r.next_id = 1;
      r.n_free = O;
      r.n_cfree = CP;
      r.kf_first = 1;
      r.kf_last_changed = 1 << 30;
      r.w_th_t = r.w_full_t = -1e300;
      r.w_dirty = 1;
    }
    CK(cudaMemcpy(B.maps, maps.data(), sizeof(MapRec) * M, cudaMemcpyHostToDevice));
    std::vector<int32_t> fl(MO);
    for (int m = 0; m < M; ++m)
      for (int i = 0; i < O; ++i) fl[(size_t)m * O + i] = O - 1 - i;   // pop order 0, 1, 2, ...
    CK(cudaMemcpy(B.freel, fl.data(), sizeof(int32_t) * MO, cudaMemcpyHostToDevice));
    std::vector<int32_t> cfl(MC);
    for (int m = 0; m < M; ++m)
      for (int i = 0; i < CP; ++i) cfl[(size_t)m * CP + i] = CP - 1 - i;   // pop order 0, 1, 2, ...
    CK(cudaMemcpy(B.cfreel, cfl.data(), sizeof(int32_t) * MC, cudaMemcpyHostToDevice));
    std::vector<CloudRec> cl(MC);
    for (auto& c : cl) { memset(&c, 0, sizeof(c)); c.vgen = 1; c.cgen = 1; c.cver = 0xffffffffu; }
    CK(cudaMemcpy(B.clouds, cl.data(), sizeof(CloudRec) * MC, cudaMemcpyHostToDevice));
    const std::vector<int32_t>& need = need_table();
    CK(cudaMemcpy(B.need_tab, need.data(), sizeof(int32_t) * need.size(), cudaMemcpyHostToDevice));
    // export8 / probability LUTs (grid.cpp:118-123)
    std::vector<int8_t> l8(nlut);
    std::vector<float> lp(nlut);
    for (int k = 0; k < nlut; ++k) {
      const float L = float(k - B.lut_off) / 256;
      const float pr = 1.f / (1.f + std::exp(-L));
      lp[k] = pr;
      l8[k] = (int8_t)std::lround(100.f * pr);
    }
    CK(cudaMemcpy(B.lut8, l8.data(), nlut, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(B.lutp, lp.data(), sizeof(float) * nlut, cudaMemcpyHostToDevice));
    // free-ray bin directions (scan.cpp:435-437)
    std::vector<float> bc(p->bins), bsn(p->bins);
    const float bin_scale = p->bins / (2.f * float(M_PI));
    for (int k = 0; k < p->bins; ++k) {
      const float a = (k + 0.5f) / bin_scale - float(M_PI);
      bc[k] = std::cos(a);
      bsn[k] = std::sin(a);
    }
    CK(cudaMemcpy(B.bin_cos, bc.data(), sizeof(float) * p->bins, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(B.bin_sin, bsn.data(), sizeof(float) * p->bins, cudaMemcpyHostToDevice));
  }
  k_fill_d<<<256, 256>>>(B.vfirst, (size_t)M * B.view_slots * SMG_VIEW_BANDS, -1e300);
  k_fill_i64<<<256, 256>>>(B.vkey, (size_t)M * B.view_slots, INT64_MIN);
  k_fill_i8<<<256, 256>>>(B.gc8, G, (int8_t)-1);
  b->launches += 3;
  CK(cudaGetLastError());
  CK(cudaMallocHost(&b->h_ring, sizeof(FrameDev) * M * smg_batch::kRing));
  for (int r = 0; r < smg_batch::kRing; ++r) CK(cudaEventCreateWithFlags(&b->ring_ev[r], cudaEventDisableTiming));
  {
    const char* ge = getenv("SMG_STREAM_GROUPS");   // maps per launch = M / groups
    b->groups = std::max(1, std::min(smg_batch::kGroupsMax, ge ? atoi(ge) : (M >= 32 ? 4 : 1)));
    for (int g = 0; g < smg_batch::kGroupsMax; ++g) {
      if (g > 0) CK(cudaStreamCreateWithFlags(&b->s_grp[g], cudaStreamNonBlocking));
      CK(cudaStreamCreateWithFlags(&b->s_gridg[g], cudaStreamNonBlocking));
      for (cudaEvent_t* e : {&b->ev_fork[g], &b->ev_join[g], &b->ev_copied[g], &b->ev_gdone[g], &b->ev_dma[g], &b->ev_wall[g]})
        CK(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    }
    {   // host-input streams; SMG_COPY_PRIORITY=1 gives them the highest priority (the SMs' reads of
        // pinned host frames then get SMs ahead of the previous keyframe's chain)
      int lo = 0, hi = 0;
      CK(cudaDeviceGetStreamPriorityRange(&lo, &hi));
      const char* pe = getenv("SMG_COPY_PRIORITY");
      const int pr = pe && atoi(pe) != 0 ? hi : lo;
      CK(cudaStreamCreateWithPriority(&b->s_copy, cudaStreamNonBlocking, pr));
      CK(cudaStreamCreateWithPriority(&b->s_dma, cudaStreamNonBlocking, pr));
    }
    CK(cudaEventCreateWithFlags(&b->ev_up, cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&b->ev_done, cudaEventDisableTiming));
    CK(cudaEventRecord(b->ev_done, 0));
    for (int s2 = 0; s2 < 2; ++s2) {
      CK(cudaEventCreateWithFlags(&b->ev_set[s2], cudaEventDisableTiming));
      CK(cudaEventRecord(b->ev_set[s2], 0));
    }
  }
  b->last_cam_t.assign(M, -1e300);
  b->last_cam_fwd.assign(3 * (size_t)M, 0.0);
  b->h_closed.assign(2 * (size_t)M, 0);
  b->h_tried.assign(2 * (size_t)M, 0);
  b->h_gref.assign(2 * (size_t)M, 0.0);
  b->h_gref_t.assign(2 * (size_t)M, -1e300);
  // kernels with large dynamic shared memory
  CK(cudaFuncSetAttribute(k_obs, cudaFuncAttributeMaxDynamicSharedMemorySize, OBS_SMEM));
  {
    const int sm_assoc = ((D * 4 + SP_MAX * 12 + 7) & ~7) + O * 8;
    CK(cudaFuncSetAttribute(k_assoc, cudaFuncAttributeMaxDynamicSharedMemorySize, sm_assoc));
    CK(cudaFuncSetAttribute(k_merge_gate, cudaFuncAttributeMaxDynamicSharedMemorySize, MP_SMEM(O)));
    CK(cudaFuncSetAttribute(k_relink, cudaFuncAttributeMaxDynamicSharedMemorySize, 3 * 8 * RELINK_STAGE));
    CK(cudaFuncSetAttribute(k_update, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)UPD_SMEM(B)));
    CK(cudaFuncSetAttribute(k_struct, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)STRUCT_SMEM));
    CK(cudaFuncSetAttribute(k_reenc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)RE_SMEM(B)));
  }
  CK(cudaDeviceSynchronize());
  *out = b;
  return SMG_OK;
}

// ObjFrame::depth_mm: every reference reader takes mm * 1e-3f (objmap.cpp:227, :269, :677,
// :1400, scan.cpp:120); the chain reads the same floats from the staging image
__global__ void k_depth_mm(Batch B) {
  const int m = B.map0 + blockIdx.y;
  const FrameDev& F = B.frames[m];
  if (!F.active || !F.depth_mm) return;
  const size_t n = (size_t)F.w * F.h;
  float* out = const_cast<float*>(F.depth);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    out[i] = (float)F.depth_mm[i] * 1e-3f;
}

__global__ void k_begin(Batch B) {
  const int m = B.map0 + blockIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active) return;
  for (int k = threadIdx.x; k < B.max_det; k += blockDim.x) {
    AssocRec& a = B.assoc[(size_t)m * B.max_det + k];
    a.obj_id = 0; a.n_valid = 0; a.area_px = 0; a.depth_med = 0;
  }
  if (F.wall_set && !B.walls_on) {   // ObjectMap::wsegs_ = this keyframe's wall segments (objmap.cpp:534)
    const int nw = min(F.n_wseg, SMG_WALL_SEGS_MAX);
    double* dst = B.wsegs + (size_t)m * SMG_WALL_SEGS_MAX * 4;
    for (int i = threadIdx.x; i < 4 * nw; i += blockDim.x) dst[i] = F.wsegs[i];
  }
  if (threadIdx.x == 0) {
    MapRec* R = &B.maps[m];
    if (F.wall_set && !B.walls_on) R->n_wseg = min(F.n_wseg, SMG_WALL_SEGS_MAX);
    R->wfr = F.wall_set && !B.walls_on ? min(F.n_wseg, SMG_WALL_SEGS_MAX) : 0;   // extracted ones: k_walls
    R->n_events = 0;
    R->n_evn = 0;
    R->n_obs = 0;
    R->n_pts = 0;
    R->n_vnew = 0;
    R->n_targets = 0;
    if (!B.reenc_on) R->re_n = 0;
    B.mcand_n[m] = 0;
    B.mgl_n[m] = 0;
    B.mgl_n[B.M + m] = 0;
  }
}

// The keyframe chain of one group of maps (B.map0 .. B.map0 + Mg - 1) on stream st, with the
// occupancy kernel on the side stream sgrid (forked after k_begin, joined at the end).
// dynamic shared memory of the text-model kernels
#define RN_CTAS 8
static size_t rn_smem(const Batch& B) { return (size_t)RN_WARPS * 2 * B.txt.n_labels * sizeof(double); }
static size_t obt_smem(const Batch& B) { return ((size_t)B.D + B.txt.n_labels) * sizeof(float); }
static size_t wv_smem(const Batch& B) { return B.text_on ? ((size_t)B.D + 2 * B.txt.n_labels) * sizeof(float) : 0; }

static int launch_group(smg_batch* b, const Batch& B, int Mg, cudaStream_t st, cudaStream_t sgrid, cudaEvent_t efork,
                        cudaEvent_t ejoin, cudaEvent_t ewall) {
  { cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
  k_begin<<<Mg, 128, 0, st>>>(B);
  if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after launch ") + std::to_string(b->dbg_last) + ": " + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } ++b->dbg_last; }
  if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({0, {e0, e1}}); } }
  if (B.walls_on) {   // the ignore footprints, from the objects as they were before this keyframe
    cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
    k_wall_rects<<<Mg, 256, 0, st>>>(B);
    ++b->launches;
    if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after k_wall_rects: ") + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } }
    if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({17, {e0, e1}}); }
  }
  if (b->hands_on) {
    cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
    k_hands<<<Mg, HANDS_THREADS, 0, st>>>(B);
    ++b->launches;
    if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after k_hands: ") + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } }
    if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({15, {e0, e1}}); }
  }
  // fork: the occupancy grid (Mapper2D::keyframe) is independent of the object chain
  CK(cudaEventRecord(efork, st));
  CK(cudaStreamWaitEvent(sgrid, efork, 0));
  { cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, sgrid); }
  k_grid<<<Mg, GRID_THREADS, 0, sgrid>>>(B);
  if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(sgrid); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after k_grid: ") + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } }
  if (b->timing) { cudaEventRecord(e1, sgrid); b->ev_used.push_back({13, {e0, e1}}); } }
  if (B.walls_on) {   // wall segments of the updated grid, before the observations read them
    cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, sgrid); }
    k_walls<<<Mg, WALL_THREADS, WALL_SMEM, sgrid>>>(B);
    ++b->launches;
    if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(sgrid); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after k_walls: ") + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } }
    if (b->timing) { cudaEventRecord(e1, sgrid); b->ev_used.push_back({17, {e0, e1}}); }
    CK(cudaEventRecord(ewall, sgrid));
  }
  CK(cudaEventRecord(ejoin, sgrid));
  { cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
  k_merge_gate<<<dim3(MP_CTAS, Mg), 256, MP_SMEM(B.O), st>>>(B);
  k_merge_pairs<<<dim3(MP_CTAS, Mg), 256, 0, st>>>(B);   // timed together with k_merge_gate
  if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after launch ") + std::to_string(b->dbg_last) + ": " + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } ++b->dbg_last; }
  if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({1, {e0, e1}}); } }
  { cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
  k_merge_apply<<<Mg, 512, 0, st>>>(B);
  if (B.text_on) { k_rename<<<dim3(RN_CTAS, Mg), RN_WARPS * 32, rn_smem(B), st>>>(B); ++b->launches; }   // merged objects
  if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after launch ") + std::to_string(b->dbg_last) + ": " + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } ++b->dbg_last; }
  if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({2, {e0, e1}}); } }
  if (B.walls_on) CK(cudaStreamWaitEvent(st, ewall, 0));
  { cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
  k_obs<<<dim3(B.max_det, Mg), OBS_THREADS, OBS_SMEM, st>>>(B);
  if (B.text_on) { k_obs_text<<<dim3(B.max_det, Mg), OBT_THREADS, obt_smem(B), st>>>(B); ++b->launches; }
  if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after launch ") + std::to_string(b->dbg_last) + ": " + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } ++b->dbg_last; }
  if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({3, {e0, e1}}); } }
  { cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
  k_obs_finalize<<<Mg, 32, 0, st>>>(B);
  if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after launch ") + std::to_string(b->dbg_last) + ": " + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } ++b->dbg_last; }
  if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({4, {e0, e1}}); } }
  { cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
  k_assoc<<<dim3(B.max_det, Mg), ASSOC_THREADS, ((B.D * 4 + SP_MAX * 12 + 7) & ~7) + B.O * 8, st>>>(B);
  if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after launch ") + std::to_string(b->dbg_last) + ": " + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } ++b->dbg_last; }
  if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({5, {e0, e1}}); } }
  { cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
  k_update<<<Mg, UPD_THREADS, UPD_SMEM(B), st>>>(B);
  k_update_vec<<<dim3(B.max_det, Mg), UPD_THREADS, 0, st>>>(B);   // timed together with k_update
  if (B.text_on) { k_rename<<<dim3(RN_CTAS, Mg), RN_WARPS * 32, rn_smem(B), st>>>(B); ++b->launches; }   // objects seen
  if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after launch ") + std::to_string(b->dbg_last) + ": " + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } ++b->dbg_last; }
  if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({6, {e0, e1}}); } }
  { cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
  k_absent<<<dim3(4, Mg), 256, 0, st>>>(B);
  if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after launch ") + std::to_string(b->dbg_last) + ": " + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } ++b->dbg_last; }
  if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({7, {e0, e1}}); } }
  { cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
  k_relink<<<Mg, 256, 3 * 8 * RELINK_STAGE, st>>>(B);
  if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after launch ") + std::to_string(b->dbg_last) + ": " + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } ++b->dbg_last; }
  if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({8, {e0, e1}}); } }
  { cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
  k_struct<<<dim3(STRUCT_CTAS, Mg), 256, STRUCT_SMEM, st>>>(B);
  if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after launch ") + std::to_string(b->dbg_last) + ": " + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } ++b->dbg_last; }
  if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({9, {e0, e1}}); } }
  { cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
  k_prune<<<Mg, 256, 0, st>>>(B);
  if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after launch ") + std::to_string(b->dbg_last) + ": " + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } ++b->dbg_last; }
  if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({10, {e0, e1}}); } }
  { cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
  k_markview<<<dim3(MV_CTAS, Mg), 256, 0, st>>>(B);
  if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after launch ") + std::to_string(b->dbg_last) + ": " + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } ++b->dbg_last; }
  if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({11, {e0, e1}}); } }
  { cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
  k_cloud_add<<<dim3(WORK_SLOTS, Mg), 512, 0, st>>>(B);
  if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after launch ") + std::to_string(b->dbg_last) + ": " + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } ++b->dbg_last; }
  if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({12, {e0, e1}}); } }
  if (b->views_alloc) {   // best views of the keyframe (capi.cpp:903-998); none exist before the first image
    cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
    k_views_pick<<<Mg, VIEW_THREADS, 0, st>>>(B);
    if (b->views_push) k_views_crop<<<dim3(B.max_det, Mg), VCROP_THREADS, 0, st>>>(B);
    b->launches += b->views_push ? 2 : 1;
    if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after k_views: ") + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } }
    if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({16, {e0, e1}}); }
  }
  if (B.reenc_on) { cudaEvent_t e0 = nullptr, e1 = nullptr; if (b->timing) { e0 = ev_get(b); e1 = ev_get(b); cudaEventRecord(e0, st); }
  k_reenc<<<dim3(RE_CTAS, Mg), RE_THREADS, RE_SMEM(B), st>>>(B);
  if (b->dbg_sync) { cudaError_t e_ = cudaStreamSynchronize(st); if (e_ == cudaSuccess) e_ = cudaGetLastError(); if (e_ != cudaSuccess) { g_err = std::string("after launch ") + std::to_string(b->dbg_last) + ": " + cudaGetErrorString(e_); return SMG_ERR_DEVICE; } ++b->dbg_last; }
  if (b->timing) { cudaEventRecord(e1, st); b->ev_used.push_back({14, {e0, e1}}); } }
  CK(cudaStreamWaitEvent(st, ejoin, 0));   // join
  b->launches += B.reenc_on ? 17 : 16;
  return SMG_OK;
}

// ObjectMap::gripGap (objmap.cpp:387-397): gripper value -> finger gap, piecewise linear
static double grip_gap(const smg_params& P, double g) {
  const int n = P.n_grip_gap;
  if (n <= 0) return 0;
  if (g <= P.grip_gap[0][0]) return P.grip_gap[0][1];
  for (int i = 1; i < n; ++i)
    if (g <= P.grip_gap[i][0]) {
      const double a = (g - P.grip_gap[i - 1][0]) / std::max(1e-12, P.grip_gap[i][0] - P.grip_gap[i - 1][0]);
      return P.grip_gap[i - 1][1] + a * (P.grip_gap[i][1] - P.grip_gap[i - 1][1]);
    }
  return P.grip_gap[n - 1][1];
}

// Best-view records and image slots, and the RGBA staging of host frames: allocated by the first
// push that carries an RGBA image (one allocation for the batch's life, not per frame).
static int views_alloc(smg_batch* b, bool host) {
  Batch& B = b->B;
  const size_t MD = (size_t)B.M * B.max_det;
  if (!b->views_alloc) {
    if (int r = dalloc(b, &B.vrec, MD)) return r;
    if (int r = dalloc(b, &B.vrgb, MD * VIEW_PIX * 3)) return r;
    if (int r = dalloc(b, &B.vdepth, MD * VIEW_PIX)) return r;
    if (int r = dalloc(b, &B.vmask, MD * VIEW_PIX)) return r;
    b->views_alloc = true;
  }
  if (host && !b->d_rgba)
    if (int r = dalloc(b, &b->d_rgba, 2 * (size_t)B.M * b->max_w * b->max_h * 4)) return r;
  return SMG_OK;
}

int smg_push_frames(smg_batch* b, const smg_frame* frames, int n, int where, void* stream) {
  if (!b || !frames || n <= 0 || n > b->B.M || (where != SMG_MEM_DEVICE && where != SMG_MEM_HOST))
    return fail(SMG_ERR_ARGS, "smg_push_frames: bad arguments");
  Batch& B = b->B;
  cudaStream_t st = (cudaStream_t)stream;
  b->last_stream = st;
  CK(cudaSetDevice(b->dev));
  const smg_params& P = B.p;
  for (int i = 0; i < n; ++i) {
    const smg_frame& f = frames[i];
    if (f.w <= 0 || f.h <= 0 || f.w > b->max_w || f.h > b->max_h || (!f.depth && !f.depth_mm) || f.n_det < 0 || f.n_det > B.max_det ||
        (f.n_det > 0 && (!f.box || !f.cls || (!f.mask_bits && (!f.label || !f.det_label)))) ||
        (f.emb && f.emb_dtype != SMG_EMB_F32 && f.emb_dtype != SMG_EMB_BF16))
      return fail(SMG_ERR_ARGS, "smg_push_frames: bad frame");
    if (f.mask_bits && (f.mask_w <= 0 || f.mask_h <= 0 || f.mask_w > b->max_w || f.mask_h > b->max_h || !(f.mask_sx > 0) ||
                        !(f.mask_sy > 0) || f.img_w < 0 || f.img_h < 0))
      return fail(SMG_ERR_ARGS, "smg_push_frames: bad detection mask grid (mask_w x mask_h <= max_w x max_h, scales > 0)");
    if (f.wall_segs && (f.n_wall_segs < 0 || f.n_wall_segs > SMG_WALL_SEGS_MAX))
      return fail(SMG_ERR_ARGS, "smg_push_frames: n_wall_segs must be in [0, SMG_WALL_SEGS_MAX]");
    if (f.wall_segs && B.walls_on)
      return fail(SMG_ERR_ARGS, "smg_push_frames: wall_segs given while the library extracts walls (smg_set_walls)");
  }
  {
    bool any_rgba = false, any_wall = false;
    for (int i = 0; i < n; ++i) {
      any_rgba = any_rgba || frames[i].rgba != nullptr;
      any_wall = any_wall || (frames[i].wall_segs != nullptr && frames[i].n_wall_segs > 0);
    }
    if (any_rgba)
      if (int r = views_alloc(b, where == SMG_MEM_HOST)) return r;
    if (any_wall && where == SMG_MEM_HOST && !b->h_wall) {
      const size_t per = (size_t)B.M * SMG_WALL_SEGS_MAX * 4;
      if (int r = dalloc(b, &b->d_wall, 2 * per)) return r;
      CK(cudaMallocHost(&b->h_wall, sizeof(double) * per * smg_batch::kRing));
    }
  }
  // pinned descriptor ring: wait until the copy that last read this slot has run
  b->dbg_last = 0;
  const int slot = (int)(b->n_push++ % smg_batch::kRing);
  if (b->ring_used[slot]) CK(cudaEventSynchronize(b->ring_ev[slot]));
  b->h_frames = b->h_ring + (size_t)slot * B.M;
  const size_t WH = (size_t)b->max_w * b->max_h;
  size_t emb_off = 0;   // host embeddings are staged packed, frame after frame
  // this push's staging set (the other one may still be read by the previous chain)
  const int ss = b->stage_set;
  b->stage_set ^= 1;
  float* sd_depth = b->d_depth + (size_t)ss * B.M * WH;
  uint16_t* sd_label = b->d_label + (size_t)ss * B.M * WH;
  unsigned char* sd_emb = b->d_emb + (size_t)ss * B.M * B.max_det * B.D * 4;
  uint16_t* sd_depth_mm = b->d_depth_mm + (size_t)ss * B.M * WH;
  uint32_t* sd_mask = b->d_mask + (size_t)ss * B.M * B.max_det * b->mask_words_max;
  uint8_t* sd_rgba = b->d_rgba ? b->d_rgba + (size_t)ss * B.M * WH * 4 : nullptr;
  const size_t wall_per = (size_t)B.M * SMG_WALL_SEGS_MAX * 4;
  double* sd_wall = b->d_wall ? b->d_wall + (size_t)ss * wall_per : nullptr;
  double* hs_wall = b->h_wall ? b->h_wall + (size_t)slot * wall_per : nullptr;
  size_t wall_off = 0;   // host wall segments are staged packed, frame after frame
  // Host frames in pinned (device-accessible) memory are read in place: k_gather fetches only
  // the pixels the chain reads.  Any other host memory goes through whole-frame copies.
  bool gather = where == SMG_MEM_HOST && b->host_gather && b->max_w <= GATHER_WMAX;
  for (int i = 0; i < n && gather; ++i) gather = frames[i].depth != nullptr;   // millimetre depth travels whole
  auto dev_ptr = [](const void* p, size_t bytes) -> const void* {
    cudaPointerAttributes a0, a1;
    if (cudaPointerGetAttributes(&a0, p) != cudaSuccess || cudaPointerGetAttributes(&a1, (const char*)p + bytes - 1) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    if (a0.type != cudaMemoryTypeHost || a1.type != cudaMemoryTypeHost || !a0.devicePointer || !a1.devicePointer) return nullptr;
    return a0.devicePointer;
  };
  std::vector<const void*> dh(gather ? 2 * (size_t)n : 0, nullptr);
  for (int i = 0; i < n && gather;) {
    // a run of frames that lie back to back (depth and labels) is checked at its two ends
    const size_t pi = (size_t)frames[i].w * frames[i].h;
    int j = i + 1;
    while (j < n && (size_t)frames[j].w * frames[j].h == pi && frames[j].depth == frames[i].depth + (j - i) * pi &&
           (frames[i].label ? frames[j].label == frames[i].label + (j - i) * pi : frames[j].label == nullptr))
      ++j;
    const char* d0 = (const char*)dev_ptr(frames[i].depth, (size_t)(j - i) * pi * 4);
    const char* l0 = frames[i].label ? (const char*)dev_ptr(frames[i].label, (size_t)(j - i) * pi * 2) : nullptr;
    if (!d0 || (frames[i].label && !l0)) { gather = false; break; }
    for (int k = i; k < j; ++k) {
      dh[2 * k] = d0 + (size_t)(k - i) * pi * 4;
      dh[2 * k + 1] = l0 ? l0 + (size_t)(k - i) * pi * 2 : nullptr;
    }
    i = j;
  }
  for (int m = 0; m < B.M; ++m) {
    FrameDev& d = b->h_frames[m];
    memset(&d, 0, sizeof(d));
    if (m >= n) continue;
    const smg_frame& f = frames[m];
    d.active = 1;
    d.stamp = f.stamp;
    b->last_stamp[m] = f.stamp;
    d.w = f.w;
    d.h = f.h;
    d.fx = f.fx; d.fy = f.fy; d.cx = f.cx; d.cy = f.cy;
    memcpy(d.T_mc, f.T_mc, sizeof d.T_mc);
    memcpy(d.T_bc, f.T_bc, sizeof d.T_bc);
    memcpy(d.base, f.base, sizeof d.base);
    memcpy(d.eef, f.eef, sizeof d.eef);
    memcpy(d.eef_base, f.eef_base, sizeof d.eef_base);
    d.n_det = f.n_det;
    for (int k = 0; k < f.n_det; ++k) {
      d.det_label[k] = f.det_label[k];
      for (int c = 0; c < 4; ++c) d.box[k][c] = f.box[4 * k + c];
      d.cls[k] = f.cls[k];
      d.score[k] = f.score ? f.score[k] : 1.f;
    }
    d.emb_dtype = f.emb_dtype;
    // detector image and masks (sm_detections); the label-image form has the depth grid as its
    // mask grid.  Scales as the reference computes them (objmap.cpp:635-636 float, :1377 double).
    d.img_w = f.img_w > 0 ? f.img_w : f.w;
    d.img_h = f.img_h > 0 ? f.img_h : f.h;
    d.sxu_f = float(f.w) / d.img_w;
    d.syv_f = float(f.h) / d.img_h;
    d.sxu_d = double(f.w) / d.img_w;
    d.syv_d = double(f.h) / d.img_h;
    if (f.mask_bits && f.n_det > 0) {
      d.mask_w = f.mask_w; d.mask_h = f.mask_h;
      d.mask_sx = f.mask_sx; d.mask_sy = f.mask_sy; d.mask_ox = f.mask_ox; d.mask_oy = f.mask_oy;
    } else {
      d.mask_w = f.w; d.mask_h = f.h;
      d.mask_sx = d.mask_sy = 1.f; d.mask_ox = d.mask_oy = 0.f;
    }
    d.mask_words = (int32_t)(((size_t)d.mask_w * d.mask_h + 31) / 32);
    // RGB source (capi.cpp:916): views and point colours need the detector image to be the image
    if (f.rgba) {
      d.rgba = where == SMG_MEM_DEVICE ? f.rgba : sd_rgba + (size_t)m * WH * 4;
      d.views_on = d.img_w == f.w && d.img_h == f.h;
    }
    // ObjFrame::wall_segs: a set (even an empty one) replaces the stored one; none keeps it
    if (f.wall_segs) {
      d.wall_set = 1;
      d.n_wseg = f.n_wall_segs;
      if (f.n_wall_segs > 0) {
        if (where == SMG_MEM_DEVICE) {
          d.wsegs = f.wall_segs;
        } else {
          memcpy(hs_wall + wall_off, f.wall_segs, sizeof(double) * 4 * f.n_wall_segs);
          d.wsegs = sd_wall + wall_off;
          wall_off += 4 * (size_t)f.n_wall_segs;
        }
      }
    }
    if (where == SMG_MEM_DEVICE) {
      d.depth = f.depth ? f.depth : sd_depth + (size_t)m * WH;   // millimetres: converted into staging
      d.depth_mm = f.depth ? nullptr : f.depth_mm;
      d.label = f.label;
      d.emb = f.emb;
      d.mask_bits = f.n_det > 0 ? f.mask_bits : nullptr;
    } else {
      d.depth = sd_depth + (size_t)m * WH;
      d.depth_mm = f.depth ? nullptr : sd_depth_mm + (size_t)m * WH;
      d.label = sd_label + (size_t)m * WH;
      if (gather) {
        d.depth_host = (const float*)dh[2 * m];
        d.label_host = (const uint16_t*)dh[2 * m + 1];
      }
      d.emb = f.emb && f.n_det > 0 ? (const void*)(sd_emb + emb_off) : nullptr;
      if (d.emb) emb_off += (size_t)f.n_det * B.D * (f.emb_dtype == SMG_EMB_BF16 ? 2 : 4);
      d.mask_bits = f.mask_bits && f.n_det > 0 ? sd_mask + (size_t)m * B.max_det * b->mask_words_max : nullptr;
    }
    // host-libm scalars (objmap.cpp:520-531, bestview.cpp:77-81, grid.cpp:202)
    const double* T = f.T_mc;
    const double fwd[3] = {T[2], T[6], T[10]};
    const double dt = f.stamp - b->last_cam_t[m];
    double cam_w = 0;
    if (b->last_cam_t[m] > -1e299 && dt > 1e-6) {
      const double c = std::clamp(fwd[0] * b->last_cam_fwd[3 * m] + fwd[1] * b->last_cam_fwd[3 * m + 1] + fwd[2] * b->last_cam_fwd[3 * m + 2], -1.0, 1.0);
      cam_w = std::acos(c) / dt;
    }
    for (int k = 0; k < 3; ++k) b->last_cam_fwd[3 * m + k] = fwd[k];
    b->last_cam_t[m] = f.stamp;
    d.cam_w = cam_w;
    d.cam_steady = cam_w <= P.move_max_cam_w;
    d.blur_fac = P.kap_blur_w > 0 ? std::exp(-std::max(0.0, (double)std::max(0.f, (float)cam_w)) / P.kap_blur_w) : 1.0;
    d.cos_th = std::cos(f.base[2]);
    d.sin_th = std::sin(f.base[2]);
    // ObjectMap::updateHands' gripper state machine (objmap.cpp:448-472), host doubles like the
    // reference; the device does the object side of what it decides
    for (int h = 0; h < P.n_hands && h < 2; ++h) {
      const size_t i = 2 * (size_t)m + h;
      const float g = f.grip[h];
      const bool closed = g < P.grip_closed;
      if (b->h_gref_t[i] < -1e299 || std::fabs(g - b->h_gref[i]) > P.grip_settle_eps) { b->h_gref[i] = g; b->h_gref_t[i] = f.stamp; }
      const bool settled = f.stamp - b->h_gref_t[i] >= P.grip_settle_s - 1e-9;
      if (closed && !b->h_closed[i]) b->h_tried[i] = 0;
      const double gap = grip_gap(P, g);
      int act = 0;
      if (closed && settled && !b->h_tried[i]) {
        b->h_tried[i] = 1;
        act |= 1;
      } else if (closed && settled && gap < P.grasp_min_gap) {
        act |= 2;
      }
      if (!closed && b->h_closed[i]) act |= 4;
      b->h_closed[i] = closed;
      d.hand_act[h] = act;
      d.hand_gap[h] = gap;
      if (act & 1) b->hands_on = true;
    }
  }
  for (int m = 0; m < n; ++m) b->h_frames[m].hands_on = b->hands_on;
  b->views_push = false;
  for (int m = 0; m < n; ++m) b->views_push = b->views_push || b->h_frames[m].views_on;
  // Stream groups: maps [g*M/G, (g+1)*M/G) run their chain on stream g (the caller's stream
  // for g = 0), so the groups' kernels overlap; with host inputs, group g's chain starts as soon
  // as its own inputs have arrived on the copy stream.
  const int G = (b->timing || b->dbg_sync) ? 1 : std::max(1, std::min(b->groups, B.M));
  auto gbeg = [&](int g) { return (int)((long long)B.M * g / G); };
  // this push's descriptors go to the set its staging uses, on the copy stream, once the last
  // chain that read that set has finished (the previous chain may still be running)
  B.frames = b->frames_base + (size_t)ss * B.M;
  CK(cudaStreamWaitEvent(b->s_copy, b->ev_set[ss], 0));
  if (wall_off) {   // packed wall segments of host frames (the ring slot's event covers the source)
    CK(cudaMemcpyAsync(sd_wall, hs_wall, sizeof(double) * wall_off, cudaMemcpyHostToDevice, b->s_copy));
    b->h2d_host += (long long)(sizeof(double) * wall_off);
  }
  CK(cudaMemcpyAsync(B.frames, b->h_frames, sizeof(FrameDev) * B.M, cudaMemcpyHostToDevice, b->s_copy));
  if (where == SMG_MEM_HOST) b->h2d_host += (long long)(sizeof(FrameDev) * B.M);
  CK(cudaEventRecord(b->ring_ev[slot], b->s_copy));
  b->ring_used[slot] = true;
  CK(cudaEventRecord(b->ev_up, b->s_copy));
  if (where == SMG_MEM_HOST) {
    // the staging buffers are free once the previous chain is done; the gather reads the
    // descriptors uploaded above
    CK(cudaStreamWaitEvent(b->s_copy, b->ev_set[ss], 0));
    if (gather) {
      CK(cudaStreamWaitEvent(b->s_copy, b->ev_up, 0));
      CK(cudaStreamWaitEvent(b->s_dma, b->ev_set[ss], 0));
    }
    // in gather mode the copy engines move the embeddings and the whole sample rows (makeScan's
    // rows v = j * step, markView's rows v = stp/2 + j * stp) on s_dma, beside the SMs' gather
    cudaStream_t sdma = gather ? b->s_dma : b->s_copy;
    auto rows2d = [&](int i, int j, int first, int pitch) -> int {   // maps i..j-1, same size, back to back
      const int w = frames[i].w, h = frames[i].h;
      const size_t spitch = (size_t)pitch * w * 4;
      const size_t nrow = j - i > 1 ? (size_t)(j - i) * h / pitch : (size_t)(h - first + pitch - 1) / pitch;
      if (nrow == 0) return 0;
      CK(cudaMemcpy2DAsync(sd_depth + i * WH + (size_t)first * w, spitch, frames[i].depth + (size_t)first * w, spitch,
                           (size_t)w * 4, nrow, cudaMemcpyHostToDevice, sdma));
      b->h2d_host += (long long)(nrow * w * 4);
      return 0;
    };
    for (int g = 0; g < G; ++g) {
      const int m0 = std::min(gbeg(g), n), m1 = std::min(gbeg(g + 1), n);
      // depth and labels: one copy per run of maps that lie back to back in host memory
      for (int i = m0; i < m1 && !gather;) {
        const size_t pi = (size_t)frames[i].w * frames[i].h;
        int j = i + 1;
        while (j < m1 && pi == WH && (size_t)frames[j].w * frames[j].h == WH &&
               (const char*)frames[j].depth == (const char*)frames[i].depth + (j - i) * WH * 4 &&
               (const char*)frames[j].label == (const char*)frames[i].label + (j - i) * WH * 2 && frames[i].label)
          ++j;
        const size_t run = j - i > 1 ? (size_t)(j - i) * WH : pi;
        if (frames[i].depth) {
          CK(cudaMemcpyAsync(sd_depth + i * WH, frames[i].depth, run * 4, cudaMemcpyHostToDevice, b->s_copy));
          b->h2d_host += (long long)run * 4;
        } else {   // millimetres: staged, converted below
          CK(cudaMemcpyAsync(sd_depth_mm + i * WH, frames[i].depth_mm, pi * 2, cudaMemcpyHostToDevice, b->s_copy));
          b->h2d_host += (long long)pi * 2;
          j = i + 1;
        }
        if (frames[i].label && !frames[i].mask_bits) {
          CK(cudaMemcpyAsync(sd_label + i * WH, frames[i].label, run * 2, cudaMemcpyHostToDevice, b->s_copy));
          b->h2d_host += (long long)run * 2;
        }
        i = j;
      }
      for (int i = m0; i < m1; ++i)   // RGBA images: whole
        if (frames[i].rgba) {
          const size_t bytes = (size_t)frames[i].w * frames[i].h * 4;
          CK(cudaMemcpyAsync(sd_rgba + (size_t)i * WH * 4, frames[i].rgba, bytes, cudaMemcpyHostToDevice, b->s_copy));
          b->h2d_host += (long long)bytes;
        }
      for (int i = m0; i < m1; ++i)   // detector bit masks: whole planes
        if (frames[i].mask_bits && frames[i].n_det > 0) {
          const size_t bytes = (size_t)frames[i].n_det * b->h_frames[i].mask_words * 4;
          CK(cudaMemcpyAsync(sd_mask + (size_t)i * B.max_det * b->mask_words_max, frames[i].mask_bits, bytes,
                             cudaMemcpyHostToDevice, b->s_copy));
          b->h2d_host += (long long)bytes;
        }
      {   // millimetre depth -> metres (mm * 1e-3f, as every reference reader computes it)
        bool any = false;
        for (int i = m0; i < m1; ++i) any = any || !frames[i].depth;
        if (any) {
          Batch Bg = B;
          Bg.map0 = m0;
          k_depth_mm<<<dim3(64, m1 - m0), 256, 0, b->s_copy>>>(Bg);
          b->launches += 1;
        }
      }
      // embeddings: packed on the device; one copy per run that is packed on the host too
      for (int i = m0; i < m1;) {
        if (!frames[i].emb || frames[i].n_det <= 0) { ++i; continue; }
        const char* d0 = (const char*)b->h_frames[i].emb;
        const char* h0 = (const char*)frames[i].emb;
        size_t bytes = 0;
        int j = i;
        while (j < m1 && frames[j].emb && frames[j].n_det > 0 && (const char*)frames[j].emb == h0 + bytes &&
               (const char*)b->h_frames[j].emb == d0 + bytes) {
          bytes += (size_t)frames[j].n_det * B.D * (frames[j].emb_dtype == SMG_EMB_BF16 ? 2 : 4);
          ++j;
        }
        CK(cudaMemcpyAsync((void*)d0, h0, bytes, cudaMemcpyHostToDevice, sdma));
        b->h2d_host += (long long)bytes;
        i = j;
      }
      for (int i = m0; i < m1 && gather;) {
        const int w = frames[i].w, h = frames[i].h;
        const int step = std::max(1, (int)std::llround(w / 160.0)), stp = std::max(1, w / 32);
        int j = i + 1;
        while (j < m1 && (size_t)w * h == WH && frames[j].w == w && frames[j].h == h && h % step == 0 && h % stp == 0 &&
               frames[j].depth == frames[i].depth + (size_t)(j - i) * WH)
          ++j;
        if (int r = rows2d(i, j, 0, step)) return r;
        if (int r = rows2d(i, j, stp / 2, stp)) return r;
        i = j;
      }
      if (gather) CK(cudaEventRecord(b->ev_dma[g], b->s_dma));
      if (gather && gbeg(g + 1) > gbeg(g)) {   // group g's pixels, while group g-1 computes
        Batch Bg = B;
        Bg.map0 = gbeg(g);
        k_gather<<<dim3(GATHER_CTAS, gbeg(g + 1) - gbeg(g)), GATHER_THREADS, 0, b->s_copy>>>(Bg);
        b->launches += 1;
      }
      CK(cudaEventRecord(b->ev_copied[g], b->s_copy));
    }
  }
  if (where == SMG_MEM_DEVICE) {   // millimetre depth -> metres in the staging images
    bool any = false;
    for (int i = 0; i < n; ++i) any = any || !frames[i].depth;
    if (any) {
      CK(cudaStreamWaitEvent(st, b->ev_up, 0));
      k_depth_mm<<<dim3(64, n), 256, 0, st>>>(B);
      b->launches += 1;
      CK(cudaEventRecord(b->ev_up, st));
    }
  }
  for (int g = 0; g < G; ++g) {
    Batch Bg = B;
    Bg.map0 = gbeg(g);
    const int Mg = gbeg(g + 1) - gbeg(g);
    cudaStream_t sg = g == 0 ? st : b->s_grp[g];
    CK(cudaStreamWaitEvent(sg, b->ev_up, 0));   // the descriptors (and staging conversions) are in place
    CK(cudaStreamWaitEvent(sg, b->ev_done, 0));   // the previous chain (or whole-view answers) has run
    if (where == SMG_MEM_HOST) CK(cudaStreamWaitEvent(sg, b->ev_copied[g], 0));
    if (gather) CK(cudaStreamWaitEvent(sg, b->ev_dma[g], 0));
    if (Mg > 0)
      if (int r = launch_group(b, Bg, Mg, sg, b->s_gridg[g], b->ev_fork[g], b->ev_join[g], b->ev_wall[g])) return r;
    if (g > 0) {
      CK(cudaEventRecord(b->ev_gdone[g], sg));
      CK(cudaStreamWaitEvent(st, b->ev_gdone[g], 0));
    }
  }
  CK(cudaEventRecord(b->ev_done, st));
  CK(cudaEventRecord(b->ev_set[ss], st));   // the staging set is free again after this chain
  CK(cudaGetLastError());
  return SMG_OK;
}

static int sync_b(smg_batch* b) {
  CK(cudaSetDevice(b->dev));
  CK(cudaStreamSynchronize(b->last_stream));
  return SMG_OK;
}

static int read_map(smg_batch* b, int m, MapRec* R) {
  CK(cudaMemcpy(R, b->B.maps + m, sizeof(MapRec), cudaMemcpyDeviceToHost));
  return SMG_OK;
}

int smg_get_reencode(smg_batch* b, int m, smg_reenc_req* reqs, uint32_t* bits, int cap) {
  if (!b || m < 0 || m >= b->B.M || cap < 0) return fail(SMG_ERR_ARGS, "smg_get_reencode: bad arguments");
  if (int r = sync_b(b)) return r;
  const Batch& B = b->B;
  MapRec R;
  if (int r = read_map(b, m, &R)) return r;
  const int n = std::max(0, std::min(R.re_n, RE_CAND));
  const size_t ostride = ((size_t)b->max_w * b->max_h + 31) / 32;
  std::vector<uint32_t> pad(B.re_words);
  for (int r = 0; r < n && r < cap; ++r) {
    const int j = R.re_rank[r];
    if (j < 0 || j >= RE_CAND) return fail(SMG_ERR_DEVICE, "smg_get_reencode: bad rank");
    ReencRec rc;
    CK(cudaMemcpy(&rc, B.reenc + (size_t)m * RE_CAND + j, sizeof(rc), cudaMemcpyDeviceToHost));
    if (reqs) {
      smg_reenc_req& q = reqs[r];
      q.id = rc.id;
      for (int k = 0; k < 4; ++k) q.box[k] = rc.box[k];
      q.kappa = rc.kappa;
      for (int k = 0; k < 6; ++k) q.cam[k] = rc.cam[k];
      q.mask_w = rc.mask_w;
      q.mask_h = rc.mask_h;
    }
    if (bits) {   // rows padded to whole words on the device -> one row-major bit string
      const int mw = rc.mask_w, mh = rc.mask_h, wpr = (mw + 31) >> 5;
      if (mw <= 0 || mh <= 0 || (size_t)mh * wpr > B.re_words) return fail(SMG_ERR_DEVICE, "smg_get_reencode: bad mask size");
      CK(cudaMemcpy(pad.data(), B.reenc_bits + ((size_t)m * RE_CAND + j) * B.re_words, sizeof(uint32_t) * (size_t)mh * wpr,
                    cudaMemcpyDeviceToHost));
      uint32_t* o = bits + (size_t)r * ostride;
      const size_t nw = ((size_t)mw * mh + 31) / 32;
      std::fill(o, o + nw, 0u);
      // only the closing window was written (every other cell is zero)
      const int y0 = std::max(0, rc.win[0]), y1 = std::min(mh - 1, rc.win[1]);
      const int x0 = std::max(0, rc.win[2] * 32), x1 = std::min(mw - 1, rc.win[3] * 32 + 31);
      for (int y = y0; y <= y1; ++y)
        for (int x = x0; x <= x1; ++x)
          if ((pad[(size_t)y * wpr + (x >> 5)] >> (x & 31)) & 1u) {
            const size_t q = (size_t)y * mw + x;
            o[q >> 5] |= 1u << (q & 31);
          }
    }
  }
  return n;
}

int smg_get_objects(smg_batch* b, int m, smg_object* out, int cap) {
  if (!b || m < 0 || m >= b->B.M) return fail(SMG_ERR_ARGS, "smg_get_objects: bad arguments");
  if (int r = sync_b(b)) return r;
  const Batch& B = b->B;
  MapRec R;
  if (int r = read_map(b, m, &R)) return r;
  const int nr = out ? std::min(R.n_obj, cap) : 0;
  if (nr <= 0) return R.n_obj;
  // three copies whatever the object count: the list order, the object records up to the highest
  // slot in use, and the map's cloud records
  std::vector<int32_t> ord(R.n_obj);
  CK(cudaMemcpy(ord.data(), B.order + (size_t)m * B.O, sizeof(int32_t) * R.n_obj, cudaMemcpyDeviceToHost));
  int top = 0;
  for (int i = 0; i < nr; ++i) {
    if (ord[i] < 0 || ord[i] >= B.O) return fail(SMG_ERR_DEVICE, "smg_get_objects: corrupt object order");
    top = std::max(top, ord[i] + 1);
  }
  std::vector<ObjRec> objs((size_t)top);
  CK(cudaMemcpy(objs.data(), B.objs + (size_t)m * B.O, sizeof(ObjRec) * top, cudaMemcpyDeviceToHost));
  std::vector<CloudRec> clouds((size_t)B.C);
  CK(cudaMemcpy(clouds.data(), B.clouds + cglob(B, m, 0), sizeof(CloudRec) * B.C, cudaMemcpyDeviceToHost));
  for (int i = 0; i < nr; ++i) {
    const ObjRec& o = objs[(size_t)ord[i]];
    if (o.cloud_slot < 0 || o.cloud_slot >= B.C) return fail(SMG_ERR_DEVICE, "smg_get_objects: corrupt cloud slot");
    const CloudRec& c = clouds[(size_t)o.cloud_slot];
    smg_object& r = out[i];
    memset(&r, 0, sizeof(r));
    r.id = o.id;
    r.cls = o.cls;
    for (int k = 0; k < 3; ++k) {
      r.pos[k] = o.pos[k]; r.ext[k] = o.ext[k]; r.first_pos[k] = o.first_pos[k]; r.lo[k] = o.lo[k]; r.hi[k] = o.hi[k];
      r.P[k] = o.P[k]; r.cloud_org[k] = c.org[k];
    }
    r.n_obs = o.n_obs;
    r.first_seen = o.first_seen;
    r.last_seen = o.last_seen;
    r.state = o.state;
    r.confirmed = o.confirmed;
    r.moved = o.moved;
    r.misses = o.misses;
    r.n_vis_miss = o.n_vis_miss;
    r.score = o.score;
    r.max_det_z = o.max_det_z;
    r.last_kf = o.last_kf;
    r.appeared = o.appeared;
    r.cloud_n = c.n;
    r.cloud_version = c.version;
    r.ap_ver = o.ver;
    r.k_frag = o.k_frag;
    r.n_views = o.n_views;
    r.n_ap_obs = o.n_ap_obs;
    r.need_whole = o.need_whole;
    r.n_cams = o.n_cams;
    r.geo = o.geo;
    r.k_whole = o.k_whole;
    r.n_whole = o.n_whole;
    r.held_by = o.held_by;
    r.parent = o.parent;
    for (int k = 0; k < 3; ++k) r.parent_rel[k] = o.parent_rel[k];
    r.wall_like = o.wall_like;
    r.hide = o.hide;
    r.n_wall_obs = o.n_wall_obs;
    r.fw = o.fw;
  }
  return R.n_obj;
}

int smg_get_object_vectors(smg_batch* b, int m, int i, float* r_frag, uint16_t* views, float* vkappa, double* vstamp, int vcap) {
  if (!b || m < 0 || m >= b->B.M) return fail(SMG_ERR_ARGS, "smg_get_object_vectors: bad arguments");
  if (int r = sync_b(b)) return r;
  const Batch& B = b->B;
  MapRec R;
  if (int r = read_map(b, m, &R)) return r;
  if (i < 0 || i >= R.n_obj) return fail(SMG_ERR_ARGS, "smg_get_object_vectors: bad index");
  int32_t slot;
  CK(cudaMemcpy(&slot, B.order + (size_t)m * B.O + i, sizeof(int32_t), cudaMemcpyDeviceToHost));
  const size_t og = (size_t)m * B.O + slot;
  ObjRec o;
  CK(cudaMemcpy(&o, B.objs + og, sizeof(ObjRec), cudaMemcpyDeviceToHost));
  if (r_frag) CK(cudaMemcpy(r_frag, B.rfrag + og * B.D, sizeof(float) * B.D, cudaMemcpyDeviceToHost));
  const int nv = std::min(vcap, o.n_views);
  for (int v = 0; v < nv; ++v) {
    if (views) CK(cudaMemcpy(views + (size_t)v * B.D, B.views + (og * (B.topk + 1) + o.view_slot[v]) * B.D, 2 * B.D, cudaMemcpyDeviceToHost));
    if (vkappa) vkappa[v] = o.vkappa[v];
    if (vstamp) vstamp[v] = o.vstamp[v];
  }
  return nv;
}

int smg_get_object_whole(smg_batch* b, int m, int i, float* r_whole, double* k_whole) {
  if (!b || m < 0 || m >= b->B.M || i < 0) return fail(SMG_ERR_ARGS, "smg_get_object_whole: bad arguments");
  if (int r = sync_b(b)) return r;
  const Batch& B = b->B;
  MapRec R;
  if (int r = read_map(b, m, &R)) return r;
  if (i >= R.n_obj) return fail(SMG_ERR_ARGS, "smg_get_object_whole: no such object");
  int32_t slot;
  CK(cudaMemcpy(&slot, B.order + (size_t)m * B.O + i, sizeof(int32_t), cudaMemcpyDeviceToHost));
  ObjRec o;
  CK(cudaMemcpy(&o, B.objs + (size_t)m * B.O + slot, sizeof(ObjRec), cudaMemcpyDeviceToHost));
  if (k_whole) *k_whole = o.k_whole;
  if (r_whole) {
    if (o.has_whole) CK(cudaMemcpy(r_whole, B.rwhole + ((size_t)m * B.O + slot) * B.D, sizeof(float) * B.D, cudaMemcpyDeviceToHost));
    else memset(r_whole, 0, sizeof(float) * B.D);
  }
  return o.has_whole ? o.n_whole : 0;
}

int smg_get_object_cloud(smg_batch* b, int m, int i, float* xyz, uint32_t* seq, int cap) {
  if (!b || m < 0 || m >= b->B.M) return fail(SMG_ERR_ARGS, "smg_get_object_cloud: bad arguments");
  if (int r = sync_b(b)) return r;
  const Batch& B = b->B;
  MapRec R;
  if (int r = read_map(b, m, &R)) return r;
  if (i < 0 || i >= R.n_obj) return fail(SMG_ERR_ARGS, "smg_get_object_cloud: bad index");
  int32_t slot;
  CK(cudaMemcpy(&slot, B.order + (size_t)m * B.O + i, sizeof(int32_t), cudaMemcpyDeviceToHost));
  ObjRec o;
  CK(cudaMemcpy(&o, B.objs + (size_t)m * B.O + slot, sizeof(ObjRec), cudaMemcpyDeviceToHost));
  const size_t cs = cglob(B, m, o.cloud_slot);
  CloudRec c;
  CK(cudaMemcpy(&c, B.clouds + cs, sizeof(CloudRec), cudaMemcpyDeviceToHost));
  const int n = std::min(cap, c.n);
  if (n > 0 && (xyz || seq)) {
    std::vector<float4> pts(n);
    CK(cudaMemcpy(pts.data(), B.cpts + cs * B.cap, sizeof(float4) * n, cudaMemcpyDeviceToHost));
    for (int k = 0; k < n; ++k) {
      if (xyz) { xyz[3 * k] = pts[k].x; xyz[3 * k + 1] = pts[k].y; xyz[3 * k + 2] = pts[k].z; }
      if (seq) { uint32_t s; memcpy(&s, &pts[k].w, 4); seq[k] = s; }
    }
  }
  return c.n;
}

int smg_get_object_cloud_rgb(smg_batch* b, int m, int i, uint8_t* rgb, int cap) {
  if (!b || m < 0 || m >= b->B.M) return fail(SMG_ERR_ARGS, "smg_get_object_cloud_rgb: bad arguments");
  if (int r = sync_b(b)) return r;
  const Batch& B = b->B;
  MapRec R;
  if (int r = read_map(b, m, &R)) return r;
  if (i < 0 || i >= R.n_obj) return fail(SMG_ERR_ARGS, "smg_get_object_cloud_rgb: bad index");
  int32_t slot;
  CK(cudaMemcpy(&slot, B.order + (size_t)m * B.O + i, sizeof(int32_t), cudaMemcpyDeviceToHost));
  ObjRec o;
  CK(cudaMemcpy(&o, B.objs + (size_t)m * B.O + slot, sizeof(ObjRec), cudaMemcpyDeviceToHost));
  const size_t cs = cglob(B, m, o.cloud_slot);
  CloudRec c;
  CK(cudaMemcpy(&c, B.clouds + cs, sizeof(CloudRec), cudaMemcpyDeviceToHost));
  const int n = std::min(cap, c.n);
  if (n > 0 && rgb) {
    std::vector<uint32_t> col(n);
    CK(cudaMemcpy(col.data(), B.crgb + cs * B.cap, sizeof(uint32_t) * n, cudaMemcpyDeviceToHost));
    for (int k = 0; k < n; ++k)
      for (int q = 0; q < 3; ++q) rgb[3 * k + q] = (uint8_t)((col[k] >> (8 * q)) & 255u);
  }
  return c.n;
}

int smg_get_views(smg_batch* b, int m, smg_view* out, uint8_t* rgb, uint16_t* depth, uint8_t* mask, int cap) {
  if (!b || m < 0 || m >= b->B.M || cap < 0) return fail(SMG_ERR_ARGS, "smg_get_views: bad arguments");
  if (int r = sync_b(b)) return r;
  const Batch& B = b->B;
  if (!b->views_alloc) return 0;
  MapRec R;
  if (int r = read_map(b, m, &R)) return r;
  const int nv = std::min(R.n_vnew, B.max_det);
  for (int v = 0; v < nv && v < cap; ++v) {
    const int k = R.vnew[v];
    if (k < 0 || k >= B.max_det) return fail(SMG_ERR_DEVICE, "smg_get_views: corrupt view list");
    const size_t vs = (size_t)m * B.max_det + k;
    ViewRec V;
    CK(cudaMemcpy(&V, B.vrec + vs, sizeof(ViewRec), cudaMemcpyDeviceToHost));
    if (out) {
      smg_view& o = out[v];
      memset(&o, 0, sizeof(o));
      o.id = V.id;
      o.version = V.version;
      o.q = V.q;
      o.stamp = V.stamp;
      for (int c = 0; c < 4; ++c) { o.box[c] = V.box[c]; o.det_box[c] = V.det_box[c]; }
      o.mask_area = V.mask_area;
      o.depth_m = V.depth_m;
      o.score = V.score;
      for (int c = 0; c < 12; ++c) o.cam_T[c] = V.cam_T[c];
      o.w = V.w;
      o.h = V.h;
    }
    const size_t np = (size_t)V.w * V.h;
    if (np > VIEW_PIX) return fail(SMG_ERR_DEVICE, "smg_get_views: corrupt view size");
    if (rgb) CK(cudaMemcpy(rgb + (size_t)v * VIEW_PIX * 3, B.vrgb + vs * VIEW_PIX * 3, np * 3, cudaMemcpyDeviceToHost));
    if (depth) CK(cudaMemcpy(depth + (size_t)v * VIEW_PIX, B.vdepth + vs * VIEW_PIX, np * 2, cudaMemcpyDeviceToHost));
    if (mask) CK(cudaMemcpy(mask + (size_t)v * VIEW_PIX, B.vmask + vs * VIEW_PIX, np, cudaMemcpyDeviceToHost));
  }
  return nv;
}

int smg_get_assoc(smg_batch* b, int m, uint32_t* obj_id, int32_t* n_valid, float* area_px, float* depth_med, int cap) {
  if (!b || m < 0 || m >= b->B.M) return fail(SMG_ERR_ARGS, "smg_get_assoc: bad arguments");
  if (int r = sync_b(b)) return r;
  const Batch& B = b->B;
  FrameDev f;
  CK(cudaMemcpy(&f, B.frames + m, sizeof(FrameDev), cudaMemcpyDeviceToHost));
  std::vector<AssocRec> a(B.max_det);
  CK(cudaMemcpy(a.data(), B.assoc + (size_t)m * B.max_det, sizeof(AssocRec) * B.max_det, cudaMemcpyDeviceToHost));
  for (int k = 0; k < f.n_det && k < cap; ++k) {
    if (obj_id) obj_id[k] = a[k].obj_id;
    if (n_valid) n_valid[k] = a[k].n_valid;
    if (area_px) area_px[k] = a[k].area_px;
    if (depth_med) depth_med[k] = a[k].depth_med;
  }
  return f.n_det;
}

int smg_get_stats(smg_batch* b, int m, int64_t* out16) {
  if (!b || m < 0 || m >= b->B.M || !out16) return fail(SMG_ERR_ARGS, "smg_get_stats: bad arguments");
  if (int r = sync_b(b)) return r;
  MapRec R;
  if (int r = read_map(b, m, &R)) return r;
  const long long* s = &R.st.n_through;
  for (int k = 0; k < 16; ++k) out16[k] = s[k];
  return SMG_OK;
}

int smg_get_events(smg_batch* b, int m, double* t, uint32_t* id, int32_t* kind, int cap) {
  if (!b || m < 0 || m >= b->B.M) return fail(SMG_ERR_ARGS, "smg_get_events: bad arguments");
  if (int r = sync_b(b)) return r;
  MapRec R;
  if (int r = read_map(b, m, &R)) return r;
  const int n = std::min(R.n_events, SMG_MAX_EVENTS);
  std::vector<EventRec> ev(n);
  if (n) CK(cudaMemcpy(ev.data(), b->B.events + (size_t)m * SMG_MAX_EVENTS, sizeof(EventRec) * n, cudaMemcpyDeviceToHost));
  std::stable_sort(ev.begin(), ev.end(), [](const EventRec& a, const EventRec& c) { return a.key < c.key; });
  for (int k = 0; k < n && k < cap; ++k) {
    if (t) t[k] = ev[k].t;
    if (id) id[k] = ev[k].id;
    if (kind) kind[k] = ev[k].kind;
  }
  return n;
}

int smg_get_grid(smg_batch* b, int m, int16_t* L, uint8_t* seen, int8_t* c8) {
  if (!b || m < 0 || m >= b->B.M) return fail(SMG_ERR_ARGS, "smg_get_grid: bad arguments");
  if (int r = sync_b(b)) return r;
  const Batch& B = b->B;
  const size_t G = (size_t)B.gw_grid * B.gh_grid, o = (size_t)m * G;
  if (L) CK(cudaMemcpy(L, B.gL + o, 2 * G, cudaMemcpyDeviceToHost));
  if (c8) CK(cudaMemcpy(c8, B.gc8 + o, G, cudaMemcpyDeviceToHost));
  if (seen) {
    CK(cudaMemcpy(seen, B.gflags + o, G, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < G; ++i) seen[i] &= 1;
  }
  return (int)G;
}

int smg_get_keyframe(smg_batch* b, int m, int32_t* out3) {
  if (!b || m < 0 || m >= b->B.M || !out3) return fail(SMG_ERR_ARGS, "smg_get_keyframe: bad arguments");
  if (int r = sync_b(b)) return r;
  MapRec R;
  if (int r = read_map(b, m, &R)) return r;
  out3[0] = R.kf_inserted;
  out3[1] = R.kf_changed;
  out3[2] = R.kf_hits;
  return SMG_OK;
}

int smg_debug_check(smg_batch* b, uint64_t* out3) {
  if (!b || !out3) return SMG_ERR_ARGS;
  if (int r = sync_b(b)) return r;
  unsigned long long h[3];
  CK(cudaMemcpyFromSymbol(h, smg_chk, sizeof h));
  for (int k = 0; k < 3; ++k) out3[k] = h[k];
  return SMG_OK;
}

__global__ void k_assoc_ids(const AssocRec* a, uint32_t* out, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[i] = a[i].obj_id;
}

int smg_get_assoc_all_async(smg_batch* b, uint32_t* obj_id, int64_t* ticket) {
  if (!b || !obj_id || !ticket) return fail(SMG_ERR_ARGS, "smg_get_assoc_all_async: bad arguments");
  const Batch& B = b->B;
  CK(cudaSetDevice(b->dev));
  const size_t n = (size_t)B.M * B.max_det;
  if (!b->d_aids) {
    if (int r = dalloc(b, &b->d_aids, smg_batch::kReads * n)) return r;
    for (int i = 0; i < smg_batch::kReads; ++i) CK(cudaEventCreateWithFlags(&b->ev_rd[i], cudaEventDisableTiming));
  }
  const int slot = (int)(b->n_reads % smg_batch::kReads);
  if (b->n_reads >= smg_batch::kReads) CK(cudaEventSynchronize(b->ev_rd[slot]));   // the slot's last read is done
  uint32_t* d = b->d_aids + (size_t)slot * n;
  cudaStream_t st = b->last_stream;
  k_assoc_ids<<<(int)std::min<size_t>((n + 255) / 256, 1024), 256, 0, st>>>(B.assoc, d, (int)n);
  CK(cudaMemcpyAsync(obj_id, d, n * sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
  CK(cudaEventRecord(b->ev_rd[slot], st));
  *ticket = b->n_reads++;
  return SMG_OK;
}

int smg_wait_read(smg_batch* b, int64_t ticket) {
  if (!b || ticket < 0 || ticket >= b->n_reads) return fail(SMG_ERR_ARGS, "smg_wait_read: bad ticket");
  if (ticket < b->n_reads - smg_batch::kReads) return SMG_OK;   // long done: its slot was reused after it
  CK(cudaSetDevice(b->dev));
  CK(cudaEventSynchronize(b->ev_rd[ticket % smg_batch::kReads]));
  return SMG_OK;
}

int smg_get_assoc_all(smg_batch* b, uint32_t* obj_id) {
  if (!b || !obj_id) return fail(SMG_ERR_ARGS, "smg_get_assoc_all: bad arguments");
  const Batch& B = b->B;
  std::vector<AssocRec> a((size_t)B.M * B.max_det);
  CK(cudaSetDevice(b->dev));
  CK(cudaMemcpyAsync(a.data(), B.assoc, sizeof(AssocRec) * a.size(), cudaMemcpyDeviceToHost, b->last_stream));
  CK(cudaStreamSynchronize(b->last_stream));
  for (size_t i = 0; i < a.size(); ++i) obj_id[i] = a[i].obj_id;
  return SMG_OK;
}

int smg_timing_enable(smg_batch* b, int on) {
  if (!b) return SMG_ERR_ARGS;
  b->timing = on != 0;
  return SMG_OK;
}

int smg_timing_read(smg_batch* b, double* ms, int64_t* n, const char** names) {
  if (!b) return fail(SMG_ERR_ARGS, "smg_timing_read: bad arguments");
  if (int r = sync_b(b)) return r;
  for (auto& u : b->ev_used) {
    float t = 0;
    CK(cudaEventElapsedTime(&t, u.second.first, u.second.second));
    b->k_ms[u.first] += t;
    b->k_n[u.first] += 1;
    b->ev_pool.push_back(u.second.first);
    b->ev_pool.push_back(u.second.second);
  }
  b->ev_used.clear();
  for (int k = 0; k < SMG_NUM_KERNELS; ++k) {
    if (ms) ms[k] = b->k_ms[k];
    if (n) n[k] = b->k_n[k];
    if (names) names[k] = k_names[k];
    b->k_ms[k] = 0;
    b->k_n[k] = 0;
  }
  return SMG_OK;
}

int smg_error_word(smg_batch* b) {
  if (!b) return SMG_ERR_ARGS;
  if (int r = sync_b(b)) return r;
  int e = 0;
  for (int m = 0; m < b->B.M; ++m) {
    MapRec R;
    if (int r = read_map(b, m, &R)) return r;
    e |= R.err;
  }
  return e;
}

int64_t smg_kernel_launches(smg_batch* b) { return b ? b->launches : -1; }

// ------------------------------------------------------------------ batched apPlaneFit
// One CTA per point set; the set's scratch (z and horizontal-projection lists of its inliers,
// 2 doubles per point) starts at 2 * off[s] doubles.  Output row (10 doubles): ok, n[3], thick,
// inl, zmed, zlo, zhi, hspan; a set that is not fitted gets the reference's ApPlane defaults.
__global__ void __launch_bounds__(PF_THREADS) k_plane_sets(const float* xyz, const int32_t* off, int n_sets, int n_points,
                                                            double tau, const uint64_t* seeds, int max_iters,
                                                            const int32_t* need_tab, double* scr, double* out) {
  __shared__ BlockScratch bs;
  __shared__ PlaneSmem ps;
  __shared__ PlaneOut po;
  const int s = blockIdx.x;
  if (s >= n_sets) return;
  const int a = off[s], e = off[s + 1];
  double* o = out + 10 * (size_t)s;
  if (a < 0 || e < a || e > n_points) {   // malformed offsets: ok = -1
    if (threadIdx.x == 0) { o[0] = -1; for (int k = 1; k < 10; ++k) o[k] = 0; }
    return;
  }
  const int n = e - a;
  plane_fit(xyz + 3 * (size_t)a, n, tau, seeds[s], max_iters, need_tab, scr + 2 * (size_t)a, n, &ps, bs, &po);
  if (threadIdx.x == 0) {
    const double dflt[10] = {0, 0, 0, 1, 1, 0, 0, 0, 0, 0};
    if (!po.ok) {
      for (int k = 0; k < 10; ++k) o[k] = dflt[k];
    } else {
      o[0] = 1; o[1] = po.n[0]; o[2] = po.n[1]; o[3] = po.n[2]; o[4] = po.thick; o[5] = po.inl;
      o[6] = po.zmed; o[7] = po.zlo; o[8] = po.zhi; o[9] = po.hspan;
    }
  }
}

static int plane_args(const float* xyz, const int32_t* off, int n_sets, int n_points, double tau, const uint64_t* seeds,
                      int max_iters, double* out, const char* who) {
  if (!xyz || !off || !seeds || !out || n_sets <= 0 || n_points < 0 || !(tau > 0) || max_iters < 1)
    return fail(SMG_ERR_ARGS, (std::string(who) + ": bad arguments").c_str());
  if (max_iters > RANSAC_MAX)
    return fail(SMG_ERR_ARGS, (std::string(who) + ": max_iters above " + std::to_string(RANSAC_MAX)).c_str());
  return SMG_OK;
}

// Per-device RANSAC table for smg_plane_fit, allocated once and kept until exit.
static int plane_need_table(int dev, const int32_t** out) {
  static std::mutex mu;
  static std::vector<int32_t*> tabs;
  std::lock_guard<std::mutex> lk(mu);
  if ((int)tabs.size() <= dev) tabs.resize((size_t)dev + 1, nullptr);
  if (!tabs[(size_t)dev]) {
    const std::vector<int32_t>& need = need_table();
    int32_t* p = nullptr;
    CK(cudaMalloc(&p, sizeof(int32_t) * need.size()));
    CK(cudaMemcpy(p, need.data(), sizeof(int32_t) * need.size(), cudaMemcpyHostToDevice));
    tabs[(size_t)dev] = p;
  }
  *out = tabs[(size_t)dev];
  return SMG_OK;
}

int smg_plane_fit(const float* xyz, const int32_t* off, int n_sets, int n_points, double tau, const uint64_t* seeds,
                  int max_iters, double* out, void* stream) {
  if (int r = plane_args(xyz, off, n_sets, n_points, tau, seeds, max_iters, out, "smg_plane_fit")) return r;
  cudaStream_t st = (cudaStream_t)stream;
  int dev = 0;
  CK(cudaGetDevice(&dev));
  const int32_t* need = nullptr;
  if (int r = plane_need_table(dev, &need)) return r;
  double* scr = nullptr;
  CK(cudaMallocAsync(&scr, sizeof(double) * 2 * (size_t)std::max(n_points, 1), st));
  k_plane_sets<<<n_sets, PF_THREADS, 0, st>>>(xyz, off, n_sets, n_points, tau, seeds, max_iters, need, scr, out);
  const cudaError_t le = cudaGetLastError();
  CK(cudaFreeAsync(scr, st));
  CK(le);
  return SMG_OK;
}

// ------------------------------------------------------------------ standalone occupancy + CSM
int smg_occ_destroy(smg_occ* o);
struct smg_occ {
  OccDev G;
  int dev = 0;
  int max_hits = 0;
  std::vector<void*> allocs;
  // pinned staging of one call's inputs
  float2* h_pts = nullptr;
  float2* h_mn = nullptr;
  int32_t* h_n = nullptr;
  float2* h_org = nullptr;
  double* h_pose = nullptr;    // [M][5]
  double* h_pose0 = nullptr;   // [M][3]
  double* h_rot = nullptr;     // [M][n_rot][2]
  double* h_out = nullptr;     // [M][5 pose + score] readback
  int32_t* h_iout = nullptr;   // [M][2] best, changed
  cudaEvent_t staged = nullptr;
  bool staged_used = false;
  // current matcher geometry (cand_w depends on it)
  double csm_key[6] = {0, 0, 0, 0, 0, 0};
  double* d_cand_w = nullptr;
};

static int oalloc(smg_occ* o, void** p, size_t bytes, int fill) {
  void* q = nullptr;
  CK(cudaMalloc(&q, std::max<size_t>(bytes, 1)));
  o->allocs.push_back(q);
  CK(cudaMemset(q, fill, std::max<size_t>(bytes, 1)));
  *p = q;
  return SMG_OK;
}
#define OA(ptr, n, fill)                                                               \
  do {                                                                                 \
    void* q_ = nullptr;                                                                \
    int r_ = oalloc(o, &q_, sizeof(*(ptr)) * (size_t)(n), fill);                       \
    if (r_) { smg_occ_destroy(o); return r_; }                                         \
    *(void**)&(ptr) = q_;                                                              \
  } while (0)

int smg_occ_destroy(smg_occ* o) {
  if (!o) return fail(SMG_ERR_ARGS, "smg_occ_destroy: null");
  cudaSetDevice(o->dev);
  for (void* p : o->allocs) cudaFree(p);
  for (void* p : {(void*)o->h_pts, (void*)o->h_mn, (void*)o->h_n, (void*)o->h_org, (void*)o->h_pose, (void*)o->h_pose0,
                  (void*)o->h_rot, (void*)o->h_out, (void*)o->h_iout})
    if (p) cudaFreeHost(p);
  if (o->staged) cudaEventDestroy(o->staged);
  delete o;
  return SMG_OK;
}

int smg_occ_create(const smg_occ_params* p, int n_maps, int grid_w, int grid_h, int grid_x0, int grid_y0, int max_points,
                   int dev, smg_occ** out) {
  if (!p || !out || n_maps <= 0 || grid_w <= 0 || grid_h <= 0 || grid_w > 4096 || grid_h > 4096 || max_points <= 0 ||
      max_points > 65536 || !(p->res > 0) || p->l_min > 0 || p->l_max < 0)
    return fail(SMG_ERR_ARGS, "smg_occ_create: bad arguments");
  *out = nullptr;
  CK(cudaSetDevice(dev));
  smg_occ* o = new smg_occ();
  o->dev = dev;
  OccDev& G = o->G;
  memset(&G, 0, sizeof(G));
  const int M = n_maps;
  G.M = M; G.W = grid_w; G.H = grid_h; G.X0 = grid_x0; G.Y0 = grid_y0; G.res = p->res;
  // OccGrid::OccGrid (grid.cpp:8-22): fixed-point steps and the LUTs, host libm
  const int kQ = 256;
  G.q_hit = (int)std::lround(p->l_hit * kQ);
  G.q_miss = (int)std::lround(p->l_miss * kQ);
  G.q_min = (int)std::lround(p->l_min * kQ);
  G.q_max = (int)std::lround(p->l_max * kQ);
  G.lut_off = -G.q_min;
  const int nlut = G.q_max - G.q_min + 1;
  std::vector<int8_t> l8(nlut);
  std::vector<uint16_t> lq(nlut);
  for (int k = 0; k < nlut; ++k) {
    const float L = float(k - G.lut_off) / kQ;
    const float pr = 1.f / (1.f + std::exp(-L));
    l8[k] = int8_t(std::lround(100.f * pr));
    const float pc = std::min(std::max(pr, p->pmin), p->pmax);   // OccGrid::prob clamp
    lq[k] = (uint16_t)std::lround((double)pc * 65535.0);
  }
  G.q_unseen = (uint16_t)std::lround((double)p->pmin * 65535.0);
  G.max_pts = max_points;
  const size_t cells = (size_t)M * grid_w * grid_h;
  OA(G.L, cells, 0);
  OA(G.c8, cells, 0xff);
  OA(G.flags, cells, 0);
  OA(G.cold, cells, 0);
  OA(G.cnt, cells, 0);
  OA(G.touch, cells, 0xff);
  OA(G.Q, cells, 0);
  int8_t* lut8 = nullptr;
  uint16_t* qlut = nullptr;
  OA(lut8, nlut, 0);
  OA(qlut, nlut, 0);
  CK(cudaMemcpy(lut8, l8.data(), nlut, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(qlut, lq.data(), nlut * 2, cudaMemcpyHostToDevice));
  G.lut8 = lut8;
  G.qlut = qlut;
  {   // unseen cells read pmin
    std::vector<uint16_t> q0((size_t)grid_w * grid_h, G.q_unseen);
    for (int m = 0; m < M; ++m)
      CK(cudaMemcpy(G.Q + (size_t)m * grid_w * grid_h, q0.data(), q0.size() * 2, cudaMemcpyHostToDevice));
  }
  OA(G.scan_id, M, 0);
  OA(G.changed, M, 0);
  OA(G.err, M, 0);
  OA(G.pts, (size_t)M * 3 * max_points, 0);
  OA(G.mn, (size_t)M * max_points, 0);
  OA(G.nmhf, (size_t)M * 3, 0);
  OA(G.origin, M, 0);
  OA(G.pose, (size_t)M * 5, 0);
  OA(G.rot, (size_t)M * CSM_MAX_ROT * 2, 0);
  OA(G.pose0, (size_t)M * 3, 0);
  OA(G.score, (size_t)M * CSM_MAX_ROT * CSM_MAX_LIN * CSM_MAX_LIN, 0);
  OA(G.best, M, 0);
  OA(G.best_score, M, 0);
  OA(o->d_cand_w, (size_t)CSM_MAX_ROT * CSM_MAX_LIN * CSM_MAX_LIN, 0);
  G.cand_w = o->d_cand_w;
  CK(cudaMallocHost(&o->h_pts, sizeof(float2) * (size_t)M * 3 * max_points));
  CK(cudaMallocHost(&o->h_mn, sizeof(float2) * (size_t)M * max_points));
  CK(cudaMallocHost(&o->h_n, sizeof(int32_t) * (size_t)M * 3));
  CK(cudaMallocHost(&o->h_org, sizeof(float2) * M));
  CK(cudaMallocHost(&o->h_pose, sizeof(double) * (size_t)M * 5));
  CK(cudaMallocHost(&o->h_pose0, sizeof(double) * (size_t)M * 3));
  CK(cudaMallocHost(&o->h_rot, sizeof(double) * (size_t)M * CSM_MAX_ROT * 2));
  CK(cudaMallocHost(&o->h_out, sizeof(double) * (size_t)M * 6));
  CK(cudaMallocHost(&o->h_iout, sizeof(int32_t) * (size_t)M * 2));
  CK(cudaEventCreateWithFlags(&o->staged, cudaEventDisableTiming));
  CK(cudaFuncSetAttribute(k_csm_score, cudaFuncAttributeMaxDynamicSharedMemorySize, CSM_WIN_CELLS * 2));
  *out = o;
  return SMG_OK;
}

// stage the scans of the first n maps (host memory) into pinned buffers and copy them in
static int occ_stage(smg_occ* o, const smg_scan2* scans, int n, bool need_hits, cudaStream_t st) {
  OccDev& G = o->G;
  if (o->staged_used) CK(cudaEventSynchronize(o->staged));
  int mx = 0;
  for (int m = 0; m < G.M; ++m) {
    int* c = o->h_n + 3 * m;
    c[0] = c[1] = c[2] = 0;
    o->h_org[m] = make_float2(0.f, 0.f);
    if (m >= n) continue;
    const smg_scan2& s = scans[m];
    if (s.n_match < 0 || s.n_hit < 0 || s.n_free < 0 || s.n_match + s.n_hit + s.n_free > G.max_pts ||
        (s.n_match && (!s.mx || !s.my)) || (s.n_hit && (!s.hx || !s.hy)) || (s.n_free && (!s.fx || !s.fy)))
      return fail(SMG_ERR_ARGS, "smg_occ: bad scan (counts, pointers or more than max_points points)");
    c[0] = s.n_match; c[1] = s.n_hit; c[2] = s.n_free;
    o->h_org[m] = make_float2(s.ox, s.oy);
    float2* P = o->h_pts + (size_t)m * 3 * G.max_pts;
    float2* N = o->h_mn + (size_t)m * G.max_pts;
    for (int k = 0; k < s.n_match; ++k) {
      P[k] = make_float2(s.mx[k], s.my[k]);
      N[k] = (s.mnx && s.mny) ? make_float2(s.mnx[k], s.mny[k]) : make_float2(0.f, 0.f);
    }
    for (int k = 0; k < s.n_hit; ++k) P[s.n_match + k] = make_float2(s.hx[k], s.hy[k]);
    for (int k = 0; k < s.n_free; ++k) P[s.n_match + s.n_hit + k] = make_float2(s.fx[k], s.fy[k]);
    mx = std::max(mx, s.n_hit);
  }
  (void)need_hits;
  o->max_hits = mx;
  for (int m = 0; m < G.M; ++m) {
    const int* c = o->h_n + 3 * m;
    const size_t np = (size_t)(c[0] + c[1] + c[2]);
    if (np) CK(cudaMemcpyAsync(G.pts + (size_t)m * 3 * G.max_pts, o->h_pts + (size_t)m * 3 * G.max_pts, np * sizeof(float2),
                               cudaMemcpyHostToDevice, st));
    if (c[0]) CK(cudaMemcpyAsync(G.mn + (size_t)m * G.max_pts, o->h_mn + (size_t)m * G.max_pts, (size_t)c[0] * sizeof(float2),
                                 cudaMemcpyHostToDevice, st));
  }
  CK(cudaMemcpyAsync(G.nmhf, o->h_n, sizeof(int32_t) * 3 * G.M, cudaMemcpyHostToDevice, st));
  CK(cudaMemcpyAsync(G.origin, o->h_org, sizeof(float2) * G.M, cudaMemcpyHostToDevice, st));
  return SMG_OK;
}

static int occ_matcher_setup(smg_occ* o, const smg_csm_params* c, const double* pose0, int n, cudaStream_t st) {
  OccDev& G = o->G;
  if (!c || !(c->linear_step > 0) || !(c->angular_step > 0) || c->linear_window < 0 || c->angular_window < 0)
    return fail(SMG_ERR_ARGS, "smg_occ: bad matcher parameters");
  const int lh = (int)std::lround(c->linear_window / c->linear_step), ah = (int)std::lround(c->angular_window / c->angular_step);
  if (2 * lh + 1 > CSM_MAX_LIN || 2 * ah + 1 > CSM_MAX_ROT)
    return fail(SMG_ERR_ARGS, "smg_occ: search window too large (at most 13 offsets per axis and 81 rotations)");
  if (std::fabs(c->linear_step - (double)G.res) > 1e-6 * (double)G.res)
    return fail(SMG_ERR_ARGS, "smg_occ: linear_step must equal the grid resolution (offsets are whole cells)");
  G.lin_half = lh;
  G.n_lin = 2 * lh + 1;
  G.n_rot = 2 * ah + 1;
  G.lin_step = (double)G.res;
  G.ang_step = c->angular_step;
  const double key[6] = {(double)lh, (double)ah, c->angular_step, c->translation_weight, c->rotation_weight, (double)G.res};
  if (memcmp(key, o->csm_key, sizeof key) != 0) {
    // candidate weights exp(-(|t| w_t + |dth| w_r)^2), host libm, candidate order (j, kx, ky)
    std::vector<double> w((size_t)G.n_rot * G.n_lin * G.n_lin);
    for (int j = 0; j < G.n_rot; ++j)
      for (int kx = -lh; kx <= lh; ++kx)
        for (int ky = -lh; ky <= lh; ++ky) {
          const double t = std::hypot((double)kx * G.lin_step, (double)ky * G.lin_step);
          const double a = std::fabs((double)(j - ah) * c->angular_step);
          const double e = t * c->translation_weight + a * c->rotation_weight;
          w[((size_t)j * G.n_lin + (kx + lh)) * G.n_lin + (ky + lh)] = std::exp(-(e * e));
        }
    CK(cudaMemcpy(o->d_cand_w, w.data(), sizeof(double) * w.size(), cudaMemcpyHostToDevice));
    memcpy(o->csm_key, key, sizeof key);
  }
  for (int m = 0; m < G.M; ++m) {
    const double* P = m < n ? pose0 + 3 * m : nullptr;
    for (int k = 0; k < 3; ++k) o->h_pose0[3 * m + k] = P ? P[k] : 0.0;
    for (int j = 0; j < G.n_rot; ++j) {
      const double th = o->h_pose0[3 * m + 2] + (double)(j - ah) * c->angular_step;
      o->h_rot[((size_t)m * G.n_rot + j) * 2] = std::cos(th);
      o->h_rot[((size_t)m * G.n_rot + j) * 2 + 1] = std::sin(th);
    }
  }
  CK(cudaMemcpyAsync(G.pose0, o->h_pose0, sizeof(double) * 3 * G.M, cudaMemcpyHostToDevice, st));
  CK(cudaMemcpyAsync(G.rot, o->h_rot, sizeof(double) * 2 * G.n_rot * G.M, cudaMemcpyHostToDevice, st));
  return SMG_OK;
}

static int occ_launch_match(smg_occ* o, cudaStream_t st) {
  OccDev& G = o->G;
  const int sectors = std::max(CSM_SECTORS, (o->max_hits + 1023) / 1024);
  k_csm_score<<<dim3(sectors, G.n_rot, G.M), OCC_THREADS, CSM_WIN_CELLS * 2, st>>>(G);
  k_csm_best<<<G.M, OCC_THREADS, 0, st>>>(G);
  CK(cudaGetLastError());
  return SMG_OK;
}

static int occ_launch_insert(smg_occ* o, cudaStream_t st) {
  OccDev& G = o->G;
  int mx = 0;
  for (int m = 0; m < G.M; ++m) mx = std::max(mx, o->h_n[3 * m] + o->h_n[3 * m + 1] + o->h_n[3 * m + 2]);
  const int blocks = std::max(1, std::min(64, (mx + 63) / 64));
  k_occ_begin<<<(G.M + 127) / 128, 128, 0, st>>>(G);
  k_occ_keys<<<dim3(blocks, G.M), OCC_THREADS, 0, st>>>(G);
  k_occ_apply<<<dim3(blocks, G.M), OCC_THREADS, 0, st>>>(G);
  CK(cudaGetLastError());
  return SMG_OK;
}

static int occ_finish(smg_occ* o, int n, double* pose_out, int32_t* index_out, double* score_out, int32_t* changed_out,
                      cudaStream_t st) {
  OccDev& G = o->G;
  CK(cudaEventRecord(o->staged, st));
  o->staged_used = true;
  if (!pose_out && !index_out && !score_out && !changed_out) return SMG_OK;
  // readback: h_out = [M][5] poses then [M] scores; h_iout = [M] best then [M] changed
  CK(cudaMemcpyAsync(o->h_out, G.pose, sizeof(double) * 5 * G.M, cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(o->h_out + 5 * G.M, G.best_score, sizeof(double) * G.M, cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(o->h_iout, G.best, sizeof(int32_t) * G.M, cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(o->h_iout + G.M, G.changed, sizeof(int32_t) * G.M, cudaMemcpyDeviceToHost, st));
  std::vector<int32_t> err(G.M);
  CK(cudaMemcpyAsync(err.data(), G.err, sizeof(int32_t) * G.M, cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  for (int m = 0; m < n; ++m) {
    if (pose_out) for (int k = 0; k < 3; ++k) pose_out[3 * m + k] = o->h_out[5 * m + k];
    if (index_out) index_out[m] = o->h_iout[m];
    if (score_out) score_out[m] = o->h_out[5 * G.M + m];
    if (changed_out) changed_out[m] = err[m] ? -1 : o->h_iout[G.M + m];
  }
  return SMG_OK;
}

int smg_occ_insert(smg_occ* o, const smg_scan2* scans, const double* poses, int n, int32_t* changed_out, void* stream) {
  if (!o || !scans || !poses || n <= 0 || n > o->G.M) return fail(SMG_ERR_ARGS, "smg_occ_insert: bad arguments");
  CK(cudaSetDevice(o->dev));
  cudaStream_t st = (cudaStream_t)stream;
  if (int r = occ_stage(o, scans, n, false, st)) return r;
  OccDev& G = o->G;
  for (int m = 0; m < G.M; ++m) {   // the insert pose and its host-libm cos/sin (grid.cpp:201)
    double* q = o->h_pose + 5 * m;
    const double* P = m < n ? poses + 3 * m : nullptr;
    q[0] = P ? P[0] : 0; q[1] = P ? P[1] : 0; q[2] = P ? P[2] : 0;
    q[3] = std::cos(q[2]); q[4] = std::sin(q[2]);
  }
  CK(cudaMemcpyAsync(G.pose, o->h_pose, sizeof(double) * 5 * G.M, cudaMemcpyHostToDevice, st));
  if (int r = occ_launch_insert(o, st)) return r;
  return occ_finish(o, n, nullptr, nullptr, nullptr, changed_out, st);
}

int smg_occ_match(smg_occ* o, const smg_scan2* scans, const double* pose0, const smg_csm_params* c, int n, double* pose_out,
                  int32_t* index_out, double* score_out, void* stream) {
  if (!o || !scans || !pose0 || n <= 0 || n > o->G.M) return fail(SMG_ERR_ARGS, "smg_occ_match: bad arguments");
  CK(cudaSetDevice(o->dev));
  cudaStream_t st = (cudaStream_t)stream;
  if (int r = occ_stage(o, scans, n, true, st)) return r;
  if (int r = occ_matcher_setup(o, c, pose0, n, st)) return r;
  if (int r = occ_launch_match(o, st)) return r;
  return occ_finish(o, n, pose_out, index_out, score_out, nullptr, st);
}

int smg_occ_track(smg_occ* o, const smg_scan2* scans, const double* pose0, const smg_csm_params* c, int n, double* pose_out,
                  int32_t* index_out, double* score_out, int32_t* changed_out, void* stream) {
  if (!o || !scans || !pose0 || n <= 0 || n > o->G.M) return fail(SMG_ERR_ARGS, "smg_occ_track: bad arguments");
  CK(cudaSetDevice(o->dev));
  cudaStream_t st = (cudaStream_t)stream;
  if (int r = occ_stage(o, scans, n, true, st)) return r;
  if (int r = occ_matcher_setup(o, c, pose0, n, st)) return r;
  if (int r = occ_launch_match(o, st)) return r;
  if (int r = occ_launch_insert(o, st)) return r;
  return occ_finish(o, n, pose_out, index_out, score_out, changed_out, st);
}

int smg_occ_get_cells(smg_occ* o, int m, int16_t* L, uint8_t* seen, int8_t* c8, uint16_t* q) {
  if (!o || m < 0 || m >= o->G.M) return fail(SMG_ERR_ARGS, "smg_occ_get_cells: bad arguments");
  CK(cudaSetDevice(o->dev));
  CK(cudaDeviceSynchronize());
  const OccDev& G = o->G;
  const size_t n = (size_t)G.W * G.H, b = (size_t)m * n;
  if (L) CK(cudaMemcpy(L, G.L + b, n * 2, cudaMemcpyDeviceToHost));
  if (c8) CK(cudaMemcpy(c8, G.c8 + b, n, cudaMemcpyDeviceToHost));
  if (q) CK(cudaMemcpy(q, G.Q + b, n * 2, cudaMemcpyDeviceToHost));
  if (seen) {
    std::vector<uint8_t> f(n);
    CK(cudaMemcpy(f.data(), G.flags + b, n, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < n; ++i) seen[i] = f[i] & 1;
  }
  return (int)n;
}

// ------------------------------------------------------------------ association stress (config 2)
struct smg_assoc {
  int dev = 0, max_det = 0, max_mem = 0, dim = 0;
  unsigned long long* stamps = nullptr;   // instrumentation (smg_assoc_stamps)
  bool stamping = false;
  float* t_best = nullptr;
  float* t_second = nullptr;
  int32_t* t_idx = nullptr;
  int32_t* err = nullptr;
  int n_sm = 148;
};

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  });
  return fn;
}

// 2D bf16 [rows][dim] K-major, box = 64 x box_rows, 128-byte swizzle, zero fill outside
static int encode_rows(CUtensorMap* m, const void* ptr, int rows, int dim, int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = tmap_encoder();
  if (!fn) return fail(SMG_ERR_DEVICE, "smg_assoc: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t gdim[2] = {(cuuint64_t)dim, (cuuint64_t)rows};
  const cuuint64_t gstr[1] = {(cuuint64_t)dim * 2};
  const cuuint32_t box[2] = {(cuuint32_t)AG_BK, (cuuint32_t)box_rows};
  const cuuint32_t est[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), gdim, gstr, box, est,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SMG_ERR_ARGS, ("smg_assoc: tensor map encoding failed (" + std::to_string((int)r) + ")").c_str());
  return SMG_OK;
}

int smg_assoc_destroy(smg_assoc* a) {
  if (!a) return fail(SMG_ERR_ARGS, "smg_assoc_destroy: null");
  cudaSetDevice(a->dev);
  cudaFree(a->t_best);
  cudaFree(a->t_second);
  cudaFree(a->t_idx);
  cudaFree(a->err);
  cudaFree(a->stamps);
  delete a;
  return SMG_OK;
}

int smg_assoc_create(int max_det, int max_mem, int dim, int dev, smg_assoc** out) {
  if (!out || max_det <= 0 || max_mem <= 0 || dim <= 0 || dim % AG_BK != 0)
    return fail(SMG_ERR_ARGS, "smg_assoc_create: bad arguments (dim must be a positive multiple of 64)");
  *out = nullptr;
  CK(cudaSetDevice(dev));
  smg_assoc* a = new smg_assoc();
  a->dev = dev; a->max_det = max_det; a->max_mem = max_mem; a->dim = dim;
  const size_t nt = 2 * ((size_t)(max_mem + AG_BN - 1) / AG_BN);   // tile halves of the persistent kernel
  if (cudaMalloc(&a->t_best, sizeof(float) * max_det * nt) != cudaSuccess ||
      cudaMalloc(&a->t_second, sizeof(float) * max_det * nt) != cudaSuccess ||
      cudaMalloc(&a->t_idx, sizeof(int32_t) * max_det * nt) != cudaSuccess || cudaMalloc(&a->err, sizeof(int32_t)) != cudaSuccess) {
    smg_assoc_destroy(a);
    return fail(SMG_ERR_DEVICE, "smg_assoc_create: out of device memory");
  }
  CK(cudaMemset(a->err, 0, sizeof(int32_t)));
  CK(cudaFuncSetAttribute(k_assoc_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, AG_SMEM));
  CK(cudaFuncSetAttribute(k_assoc_gemm_p, cudaFuncAttributeMaxDynamicSharedMemorySize, AP_SMEM));
  CK(cudaDeviceGetAttribute(&a->n_sm, cudaDevAttrMultiProcessorCount, dev));
  *out = a;
  return SMG_OK;
}

int smg_assoc_match(smg_assoc* a, const uint16_t* det, const float* det_box, int n_det, const uint16_t* mem, const float* mem_box,
                    int n_mem, float iou_min, double cos_min, int32_t* match, double* score, int32_t* certified,
                    float* scores, void* stream) {
  if (!a || !det || !det_box || !mem || !mem_box || !match || !score || !certified || n_det <= 0 || n_mem <= 0 ||
      n_det > a->max_det || n_mem > a->max_mem)
    return fail(SMG_ERR_ARGS, "smg_assoc_match: bad arguments");
  if ((((uintptr_t)det) | ((uintptr_t)mem)) & 15) return fail(SMG_ERR_ARGS, "smg_assoc_match: embeddings must be 16-byte aligned");
  CK(cudaSetDevice(a->dev));
  cudaStream_t st = (cudaStream_t)stream;
  CUtensorMap tA, tB;
  if (int r = encode_rows(&tA, det, n_det, a->dim, AG_BM)) return r;
  if (int r = encode_rows(&tB, mem, n_mem, a->dim, AG_BN)) return r;
  AssocArgs g;
  memset(&g, 0, sizeof(g));
  const int n_nt = (n_mem + AG_BN - 1) / AG_BN, n_mt = (n_det + AG_BM - 1) / AG_BM;
  g.n_det = n_det; g.n_mem = n_mem; g.dim = a->dim;
  g.n_tiles = a->stamping ? n_nt : 2 * n_nt;   // per-row partial results: tiles, or tile halves
  g.det_box = det_box; g.mem_box = mem_box; g.det = det; g.mem = mem;
  g.iou_min = iou_min; g.cos_min = cos_min;
  g.delta = (double)a->dim * std::ldexp(1.0, -22);   // > K * 2^-23 (fp32 accumulation, |z| <= 1.01)
  g.t_best = a->t_best; g.t_second = a->t_second; g.t_idx = a->t_idx;
  g.scores = scores; g.match = match; g.score = score; g.certified = certified; g.err = a->err;
  g.stamps = a->stamping ? a->stamps : nullptr;
  if (a->stamping || scores) {   // the one-tile kernel: instrumented, or writing the raw scores
    const dim3 grid(n_nt, n_mt);
    k_assoc_gemm<<<grid, AG_THREADS, AG_SMEM, st>>>(tA, tB, g);
  } else {   // persistent: one CTA per SM over all tiles, epilogue overlapped with the next MMAs
    const int grid = std::min(a->n_sm, n_nt * n_mt);
    k_assoc_gemm_p<<<grid, AP_THREADS, AP_SMEM, st>>>(tA, tB, g);
  }
  {   // programmatic dependent launch: the decide grid is scheduled while the GEMM drains
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((n_det + 7) / 8);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    CK(cudaLaunchKernelEx(&cfg, k_assoc_decide, g));
  }
  CK(cudaGetLastError());
  return SMG_OK;
}

int smg_assoc_stamps(smg_assoc* a, int enable, int64_t* out16) {
  if (!a) return fail(SMG_ERR_ARGS, "smg_assoc_stamps: null");
  CK(cudaSetDevice(a->dev));
  if (!a->stamps) {
    CK(cudaMalloc(&a->stamps, 16 * sizeof(unsigned long long)));
    CK(cudaMemset(a->stamps, 0, 16 * sizeof(unsigned long long)));
  }
  if (out16) {
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpy(out16, a->stamps, 16 * sizeof(int64_t), cudaMemcpyDeviceToHost));
  }
  a->stamping = enable != 0;
  return SMG_OK;
}

int smg_assoc_error(smg_assoc* a) {
  if (!a) return fail(SMG_ERR_ARGS, "smg_assoc_error: null");
  CK(cudaSetDevice(a->dev));
  int32_t e = 0;
  CK(cudaMemcpy(&e, a->err, sizeof(e), cudaMemcpyDeviceToHost));
  return e;
}

// ------------------------------------------------------------------ text model (apLabelLogLik, apName)
static int text_dev(const smg_text* t, TextDev* T, const char* who) {
  if (!t || t->dim <= 0 || t->n_labels <= 0 || t->n_labels > TXT_MAX_LABELS || t->rows <= 0 || !t->text || !t->row_label ||
      (!t->ls_mu) != (!t->ls_sd))
    return fail(SMG_ERR_ARGS, (std::string(who) + ": bad text model").c_str());
  T->dim = t->dim; T->n_labels = t->n_labels; T->rows = t->rows; T->text = t->text; T->row_label = t->row_label;
  T->scale = t->scale; T->bias = t->bias; T->log_prior = t->log_prior; T->ls_mu = t->ls_mu; T->ls_sd = t->ls_sd;
  T->parent = t->parent; T->object_label = t->object_label;
  return SMG_OK;
}

int smg_label_loglik(const smg_text* t, const float* z, int n, float* out, void* stream) {
  TextDev T;
  if (int r = text_dev(t, &T, "smg_label_loglik")) return r;
  if (!z || !out || n <= 0) return fail(SMG_ERR_ARGS, "smg_label_loglik: bad arguments");
  const size_t sm = sizeof(float) * ((size_t)T.dim + T.n_labels);
  if (sm > 200 * 1024) return fail(SMG_ERR_ARGS, "smg_label_loglik: dim + n_labels too large");
  if (sm > 48 * 1024) CK(cudaFuncSetAttribute(k_label_loglik, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  k_label_loglik<<<n, 256, sm, (cudaStream_t)stream>>>(T, z, n, out);
  CK(cudaGetLastError());
  return SMG_OK;
}

int smg_name(const smg_text* t, const smg_name_params* p, int n_obj, const float* L_frag, const double* lw_frag,
             const float* L_whole, const double* lw_whole, const float* L_ext, const float* L_geo, const double* size,
             float* post, int32_t* lab3, float* val3, void* stream) {
  TextDev T;
  if (int r = text_dev(t, &T, "smg_name")) return r;
  if (!p || n_obj <= 0 || !size || !post || !lab3 || !val3 || (L_frag && !lw_frag) || (L_whole && !lw_whole))
    return fail(SMG_ERR_ARGS, "smg_name: bad arguments");
  NameArgs a;
  a.n_obj = n_obj; a.whole_w = p->whole_w; a.name_wmax = p->name_wmax; a.size_w = p->size_w; a.name_tau = p->name_tau;
  a.L_frag = L_frag; a.lw_frag = lw_frag; a.L_whole = L_whole; a.lw_whole = lw_whole; a.L_ext = L_ext; a.L_geo = L_geo;
  a.size = size; a.post = post; a.lab = lab3; a.val = val3;
  const size_t sm = sizeof(double) * 2 * (size_t)T.n_labels * 8;
  if (sm > 48 * 1024) CK(cudaFuncSetAttribute(k_name, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  k_name<<<(n_obj + 7) / 8, 256, sm, (cudaStream_t)stream>>>(T, a);
  CK(cudaGetLastError());
  return SMG_OK;
}

// ------------------------------------------------------------------ plane fit, no allocation
// smg_plane_fit_noalloc runs k_plane_sets on scratch that lives in this module's own static
// device memory, for callers that must not allocate device memory while they run.  The arrays
// exist on every GPU where the library is loaded, from load until process exit.  In host code
// their names are host-side shadows, not device addresses, so the kernel receives addresses
// obtained with cudaGetSymbolAddress on the current device.
#define SMG_PF_STATIC_POINTS 65536
static __device__ __align__(256) double g_pf_scratch[2 * SMG_PF_STATIC_POINTS];   // 1 MiB
static __device__ __align__(256) int32_t g_pf_need[NEED_N * NEED_N];              // 1 MiB

struct PfStaticDevice {
  bool ready = false;
  unsigned long long ctx_id = 0;   // the context the set-up ran in (cuCtxGetId)
  double* scratch = nullptr;
  int32_t* need = nullptr;
};

// Unique id of the calling thread's current context (0 when none can be read).  A device reset
// destroys the context that held the static arrays' contents; the next context has a new id.
static unsigned long long current_ctx_id() {
  typedef CUresult (*PfnCtxGetCurrent)(CUcontext*);
  typedef CUresult (*PfnCtxGetId)(CUcontext, unsigned long long*);
  static PfnCtxGetCurrent get_cur = nullptr;
  static PfnCtxGetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
      get_cur = (PfnCtxGetCurrent)p;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
      get_id = (PfnCtxGetId)p;
  });
  CUcontext c = nullptr;
  unsigned long long id = 0;
  if (!get_cur || !get_id || get_cur(&c) != CUDA_SUCCESS || !c || get_id(c, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Once per device and context, with that device current: resolve the device addresses of the
// static arrays and fill the constant iteration table (a synchronous copy, no allocation).  The
// set-up is repeated when the device's context has changed since (after a cudaDeviceReset), so
// no stale address or empty table is used.
static int pf_static_setup(int dev, PfStaticDevice* out) {
  static std::mutex mu;
  static std::vector<PfStaticDevice> devs;
  std::lock_guard<std::mutex> lk(mu);
  if ((int)devs.size() <= dev) devs.resize((size_t)dev + 1);
  PfStaticDevice& d = devs[(size_t)dev];
  const unsigned long long ctx = current_ctx_id();
  if (!d.ready || ctx == 0 || ctx != d.ctx_id) {
    d.ready = false;
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_pf_scratch);
    if (e != cudaSuccess) return fail(SMG_ERR_DEVICE, (std::string("smg_plane_fit_noalloc: cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e)).c_str());
    d.scratch = (double*)p;
    e = cudaGetSymbolAddress(&p, g_pf_need);
    if (e != cudaSuccess) return fail(SMG_ERR_DEVICE, (std::string("smg_plane_fit_noalloc: cudaGetSymbolAddress(table): ") + cudaGetErrorString(e)).c_str());
    d.need = (int32_t*)p;
    const std::vector<int32_t>& need = need_table();
    CK(cudaMemcpyToSymbol(g_pf_need, need.data(), sizeof(int32_t) * need.size()));
    d.ctx_id = current_ctx_id();
    d.ready = true;
  }
  *out = d;
  return SMG_OK;
}

int smg_plane_fit_noalloc(const float* xyz, const int32_t* off, int n_sets, int n_points, double tau,
                          const uint64_t* seeds, int max_iters, double* out, void* stream) {
  if (int r = plane_args(xyz, off, n_sets, n_points, tau, seeds, max_iters, out, "smg_plane_fit_noalloc")) return r;
  if (n_points > SMG_PF_STATIC_POINTS)
    return fail(SMG_ERR_CAPACITY, ("smg_plane_fit_noalloc: n_points " + std::to_string(n_points) +
                                   " exceeds the static scratch limit of " + std::to_string(SMG_PF_STATIC_POINTS) +
                                   " points per call (use smg_plane_fit)").c_str());
  int dev = 0;
  CK(cudaGetDevice(&dev));
  PfStaticDevice d;
  if (int r = pf_static_setup(dev, &d)) return r;
  // Nothing in the scratch has to start at zero: every entry a set reads (its inliers' z and
  // horizontal projections) is written earlier in the same launch, so no clearing is needed.
  k_plane_sets<<<n_sets, PF_THREADS, 0, (cudaStream_t)stream>>>(xyz, off, n_sets, n_points, tau, seeds, max_iters, d.need,
                                                                  d.scratch, out);
  CK(cudaGetLastError());
  return SMG_OK;
}

// ObjectMap::addWholeView (objmap.cpp:1361-1369) for the answers of sm_set_object_embeddings
// (capi.cpp:1825-1835): entry i is applied when map maps[i]'s last keyframe requested object
// ids[i] and the object still exists, with the request's kappa and camera and the keyframe's
// stamp.  One CTA per map takes that map's entries in call order.
__global__ void __launch_bounds__(256) k_whole_views(Batch B, const int32_t* maps, const uint32_t* ids, const float* emb, int n,
                                                     const double* stamps) {
  __shared__ BlockScratch bs;
  __shared__ int s_pos, s_phys, s_zero;
  __shared__ double s_k;
  const int m = blockIdx.x, tid = threadIdx.x;
  MapRec* R = &B.maps[m];
  const ReencRec* recs = B.reenc + (size_t)m * RE_CAND;
  for (int i = 0; i < n; ++i) {
    if (maps[i] != m) continue;
    if (tid == 0) {
      s_pos = -1;
      int req = -1;
      for (int r = 0; r < R->re_n && r < RE_CAND && req < 0; ++r) {
        const int j = R->re_rank[r];
        if (j >= 0 && j < RE_CAND && recs[j].id == ids[i]) req = j;
      }
      if (req >= 0)
        for (int q = 0; q < R->n_obj; ++q)
          if (obj_at(B, m, q).id == ids[i]) { s_pos = q; break; }
      if (s_pos >= 0) {
        ObjRec& o = B.objs[oglob(B, m, slot_at(B, m, s_pos))];
        double k;
        int phys;
        ap_add_view_plan(B, o, (double)recs[req].kappa, stamps[m], recs[req].cam, &k, &phys, true);
        s_k = k;
        s_phys = phys;
        s_zero = !o.has_whole;   // r_whole starts from zeros (objprob.cpp:329)
        o.has_whole = 1;
        ++R->st.n_reenc_done;
      }
    }
    __syncthreads();
    if (s_pos >= 0) {
      const size_t og = oglob(B, m, slot_at(B, m, s_pos));
      float* rw = B.rwhole + og * B.D;
      uint16_t* vz = B.views + (og * (B.topk + 1) + s_phys) * B.D;
      const float* z = emb + (size_t)i * B.D;
      for (int q = tid; q < B.D; q += blockDim.x) {
        rw[q] = (s_zero ? 0.f : rw[q]) + (float)(s_k * (double)z[q]);
        vz[q] = ref_f2h(z[q]);
      }
      __syncthreads();
      refresh_nrm(B, og, bs);
      if (B.text_on && B.txt.dim == B.D) {   // label evidence of the whole view, then a rename
        extern __shared__ __align__(16) unsigned char wv_raw[];
        float* zs = (float*)wv_raw;
        float* best = zs + B.D;
        float* ll = best + B.txt.n_labels;
        for (int q = tid; q < B.D; q += blockDim.x) zs[q] = z[q];
        __syncthreads();
        label_loglik_block(B.txt, zs, best, ll);
        ObjRec& o = B.objs[og];
        const double w = s_k / smax(1e-6, B.p.kappa_ref);
        const bool lz = !o.has_lwhole;
        float* L = B.lwhole + og * B.txt.n_labels;
        for (int l = tid; l < B.txt.n_labels; l += blockDim.x) L[l] = (lz ? 0.f : L[l]) + (float)(w * smax((double)ll[l], -60.0));
        __syncthreads();
        if (tid == 0) {
          o.lw_whole += w;
          o.has_lwhole = 1;
          o.rename = 1;   // apRename after addWholeView (objmap.cpp:1365)
        }
      }
    }
    __syncthreads();
  }
}

int smg_set_object_embeddings(smg_batch* b, const int32_t* maps, const uint32_t* ids, const float* emb, int n, int dim, int where,
                              void* stream) {
  if (!b || n < 0 || (n > 0 && (!maps || !ids || !emb)) || dim != b->B.D || (size_t)n > (size_t)b->B.M * RE_CAND ||
      (where != SMG_MEM_DEVICE && where != SMG_MEM_HOST))
    return fail(SMG_ERR_ARGS, "smg_set_object_embeddings: bad arguments (dim must be the batch's, n <= maps * 64)");
  if (n == 0) return SMG_OK;
  CK(cudaSetDevice(b->dev));
  cudaStream_t st = (cudaStream_t)stream;
  const Batch& B = b->B;
  const int32_t* dm = maps;
  const uint32_t* di = ids;
  const float* de = emb;
  if (where == SMG_MEM_HOST) {
    for (int i = 0; i < n; ++i)
      if (maps[i] < 0 || maps[i] >= B.M) return fail(SMG_ERR_ARGS, "smg_set_object_embeddings: map index out of range");
    CK(cudaMemcpyAsync(b->d_wv_map, maps, sizeof(int32_t) * n, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(b->d_wv_id, ids, sizeof(uint32_t) * n, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(b->d_wv_emb, emb, sizeof(float) * (size_t)n * B.D, cudaMemcpyHostToDevice, st));
    dm = b->d_wv_map;
    di = b->d_wv_id;
    de = b->d_wv_emb;
  }
  CK(cudaMemcpyAsync(b->d_wv_stamp, b->last_stamp.data(), sizeof(double) * B.M, cudaMemcpyHostToDevice, st));
  // after the keyframe that made the requests (all stream groups have joined on ev_done)
  CK(cudaStreamWaitEvent(st, b->ev_done, 0));
  k_whole_views<<<B.M, 256, wv_smem(B), st>>>(B, dm, di, de, n, b->d_wv_stamp);
  if (B.text_on) {   // the objects that took a whole view are renamed (objmap.cpp:1365)
    k_rename<<<dim3(RN_CTAS, B.M), RN_WARPS * 32, rn_smem(B), st>>>(B);
    b->launches += 1;
  }
  b->launches += 1;
  CK(cudaGetLastError());
  CK(cudaEventRecord(b->ev_done, st));   // the next push's chain waits for the answers
  b->last_stream = st;
  if (where == SMG_MEM_HOST) CK(cudaStreamSynchronize(st));   // the host arrays may go away after the call
  return SMG_OK;
}

// Phase-timing counters of an instrumentation build (-DSMG_PHASE_TIMING): out[2k] = cycles
// summed over the blocks' thread 0, out[2k+1] = marks, k < 64; the counters are reset.  Returns
// SMG_ERR_UNSUPPORTED in the production build.
int smg_phase_read(uint64_t* out) {
#ifdef SMG_PHASE_TIMING
  if (!out) return fail(SMG_ERR_ARGS, "smg_phase_read: bad arguments");
  unsigned long long c[64], h[64];
  CK(cudaDeviceSynchronize());
  CK(cudaMemcpyFromSymbol(c, g_phase_cycles, sizeof c));
  CK(cudaMemcpyFromSymbol(h, g_phase_hits, sizeof h));
  for (int k = 0; k < 64; ++k) { out[2 * k] = c[k]; out[2 * k + 1] = h[k]; }
  memset(c, 0, sizeof c);
  CK(cudaMemcpyToSymbol(g_phase_cycles, c, sizeof c));
  CK(cudaMemcpyToSymbol(g_phase_hits, c, sizeof c));
  return SMG_OK;
#else
  (void)out;
  return fail(SMG_ERR_UNSUPPORTED, "smg_phase_read: not an instrumentation build (-DSMG_PHASE_TIMING)");
#endif
}


int smg_set_text_model(smg_batch* b, const smg_text* t, const uint8_t* kinds, const uint8_t* so_shape, const uint8_t* flat_ok) {
  if (!b || !t || t->n_labels <= 0 || t->n_labels > TXT_MAX_LABELS || t->rows < 0 ||
      (t->rows > 0 && (t->dim != b->B.D || !t->text || !t->row_label)))
    return fail(SMG_ERR_ARGS, "smg_set_text_model: bad arguments (0 < n_labels <= 1024; rows > 0 needs dim = emb_dim)");
  if (b->n_push > 0) return fail(SMG_ERR_ARGS, "smg_set_text_model: set the text model before the first push");
  if (b->B.txt.n_labels && b->B.txt.n_labels != t->n_labels)
    return fail(SMG_ERR_ARGS, "smg_set_text_model: the label count cannot change");
  CK(cudaSetDevice(b->dev));
  Batch& B = b->B;
  const int C = t->n_labels;
  auto up = [&](auto** dst, const auto* src, size_t n) -> int {   // device copy of a host array (null stays null)
    using T = std::remove_const_t<std::remove_pointer_t<std::remove_reference_t<decltype(src)>>>;
    if (!src || n == 0) { *dst = nullptr; return SMG_OK; }
    T* d = nullptr;
    if (int r = dalloc(b, &d, n)) return r;
    CK(cudaMemcpy(d, src, n * sizeof(T), cudaMemcpyHostToDevice));
    *dst = d;
    return SMG_OK;
  };
  TextDev T;
  memset(&T, 0, sizeof(T));
  T.dim = t->rows > 0 ? t->dim : B.D;
  T.n_labels = C;
  T.rows = t->rows;
  T.scale = t->scale;
  T.bias = t->bias;
  T.object_label = t->object_label;
  int r = 0;
  if ((r = up(&T.text, t->text, (size_t)t->rows * t->dim)) || (r = up(&T.row_label, t->row_label, (size_t)t->rows)) ||
      (r = up(&T.log_prior, t->log_prior, C)) || (r = up(&T.ls_mu, t->ls_sd ? t->ls_mu : nullptr, C)) ||
      (r = up(&T.ls_sd, t->ls_mu ? t->ls_sd : nullptr, C)) || (r = up(&T.parent, t->parent, C)) || (r = up(&T.kinds, kinds, C)) ||
      (r = up(&T.so_shape, so_shape, C)) || (r = up(&T.flat_ok, flat_ok, C)))
    return r;
  const size_t MOC = (size_t)B.M * B.O * C;
  if (!B.lfrag) {
    if ((r = dalloc(b, &B.lfrag, MOC)) || (r = dalloc(b, &B.lwhole, MOC)) || (r = dalloc(b, &B.post, MOC)) ||
        (r = dalloc(b, &B.llz, (size_t)B.M * B.max_det * C)))
      return r;
  }
  B.txt = T;
  B.text_on = t->rows > 0;
  B.kinds_on = kinds != nullptr;
  CK(cudaFuncSetAttribute(k_rename, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rn_smem(B)));
  CK(cudaFuncSetAttribute(k_obs_text, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)obt_smem(B)));
  CK(cudaFuncSetAttribute(k_whole_views, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wv_smem(B)));
  return SMG_OK;
}

int smg_get_object_name(smg_batch* b, int m, int i, float* post, int32_t* lab3, float* val3) {
  if (!b || m < 0 || m >= b->B.M || i < 0) return fail(SMG_ERR_ARGS, "smg_get_object_name: bad arguments");
  if (int r = sync_b(b)) return r;
  const Batch& B = b->B;
  MapRec R;
  if (int r = read_map(b, m, &R)) return r;
  if (i >= R.n_obj) return fail(SMG_ERR_ARGS, "smg_get_object_name: no such object");
  int32_t slot;
  CK(cudaMemcpy(&slot, B.order + (size_t)m * B.O + i, sizeof(int32_t), cudaMemcpyDeviceToHost));
  ObjRec o;
  const size_t og = (size_t)m * B.O + slot;
  CK(cudaMemcpy(&o, B.objs + og, sizeof(ObjRec), cudaMemcpyDeviceToHost));
  const int C = B.txt.n_labels;
  if (post && C) {
    if (o.has_post) CK(cudaMemcpy(post, B.post + og * C, sizeof(float) * C, cudaMemcpyDeviceToHost));
    else memset(post, 0, sizeof(float) * C);
  }
  if (lab3) { lab3[0] = o.name_lab; lab3[1] = o.top_lab; lab3[2] = o.rolled; }
  if (val3) { val3[0] = o.name_p; val3[1] = o.top_p; val3[2] = o.name_H; }
  return o.has_post ? C : 0;
}

// sm_push_image's wall extraction (capi.cpp:646-698, 866-890) before every object update.
int smg_set_walls(smg_batch* b, int on) {
  if (!b || (on != 0 && on != 1)) return fail(SMG_ERR_ARGS, "smg_set_walls: bad arguments");
  if (int r = sync_b(b)) return r;
  Batch& B = b->B;
  if (on) {
    const int w = B.gw_grid, h = B.gh_grid;
    const int D = (int)std::ceil(std::hypot((double)w, (double)h)) + 2;
    if ((size_t)2 * (2 * D + 1) * sizeof(int) > WALL_SMEM || w > 65535 || h > 65535)
      return fail(SMG_ERR_ARGS, "smg_set_walls: grid window too large for wall extraction");
    if (!B.wbits) {
      const int side = D;   // a rotated window fits: ceil(hypot(w, h)) + 1 cells a side
      const size_t O = (size_t)B.O, M = (size_t)B.M;
      const size_t nw = (w + 63) / 64, snw = (side + 63) / 64;
      const size_t rp = std::min(side / 2 + 1, WALL_ACT_MAX + 1);
      B.wscr_side = side;
      B.wbits_half = (size_t)h * nw;
      B.wbits_cb = B.wbits_half + (size_t)side * snw;
      B.wbits_stride = B.wbits_cb + (size_t)side * snw;
      B.wruns_stride = 2 * (size_t)side * rp;
      B.wscr_i_stride = (8 * O + 2 * (size_t)side + 16 + 3) & ~(size_t)3;   // int4-aligned per map
      if (int r = dalloc(b, &B.wbits, M * B.wbits_stride)) return r;
      if (int r = dalloc(b, &B.wruns, M * B.wruns_stride)) return r;
      if (int r = dalloc(b, &B.wscr_i, M * B.wscr_i_stride)) return r;
      if (int r = dalloc(b, &B.wrect, M * O * 4)) return r;
      if (int r = dalloc(b, &B.wrect_prev, M * O * 4)) return r;
      if (int r = dalloc(b, &B.wall_w, M * SMG_WALL_SEGS_MAX * 4)) return r;
      if (int r = dalloc(b, &B.wall_raw, M * SMG_WALL_SEGS_MAX * 4)) return r;
      if (int r = dalloc(b, &B.wall_tmp, M * SMG_WALL_SEGS_MAX * 4)) return r;
      if (int r = dalloc(b, &B.wall_lines, M * SMG_WALL_SEGS_MAX * WALL_RPIECES * 32)) return r;
      if (int r = dalloc(b, &B.wall_lcnt, M * SMG_WALL_SEGS_MAX)) return r;
      if (int r = dalloc(b, &b->d_wstate, (size_t)WALL_STATE_LEN)) return r;
      CK(cudaFuncSetAttribute(k_walls, cudaFuncAttributeMaxDynamicSharedMemorySize, WALL_SMEM));
    }
    // a fresh extraction state (sm_reset, capi.cpp:554-558)
    std::vector<MapRec> maps((size_t)B.M);
    CK(cudaMemcpy(maps.data(), B.maps, sizeof(MapRec) * maps.size(), cudaMemcpyDeviceToHost));
    for (MapRec& r : maps) {
      r.w_th = 0;
      r.w_th_t = r.w_full_t = -1e300;
      r.w_has = 0;
      r.w_dirty = 1;
      r.n_w = r.n_rect = r.n_rect_prev = r.w_rchg = 0;
    }
    CK(cudaMemcpy(B.maps, maps.data(), sizeof(MapRec) * maps.size(), cudaMemcpyHostToDevice));
  }
  B.walls_on = on;
  return SMG_OK;
}

int smg_get_wall_segments(smg_batch* b, int m, double* out, int cap) {
  if (!b || m < 0 || m >= b->B.M || cap < 0 || (cap > 0 && !out)) return fail(SMG_ERR_ARGS, "smg_get_wall_segments: bad arguments");
  if (int r = sync_b(b)) return r;
  MapRec R;
  if (int r = read_map(b, m, &R)) return r;
  if (!b->B.walls_on || !R.w_has) return -1;
  const int n = std::min(R.n_w, SMG_WALL_SEGS_MAX);
  if (cap > 0 && n > 0)
    CK(cudaMemcpy(out, b->B.wall_w + (size_t)m * SMG_WALL_SEGS_MAX * 4, sizeof(double) * 4 * std::min(n, cap), cudaMemcpyDeviceToHost));
  return n;
}

int smg_wall_state(smg_batch* b, int m, const double pose[3], float* out) {
  if (!b || m < 0 || m >= b->B.M || !pose || !out) return fail(SMG_ERR_ARGS, "smg_wall_state: bad arguments");
  if (int r = sync_b(b)) return r;
  MapRec R;
  if (int r = read_map(b, m, &R)) return r;
  if (!b->B.walls_on || !R.w_has) return -1;
  k_wall_state<<<1, 256, 0, b->last_stream>>>(b->B, m, pose[0], pose[1], pose[2], b->d_wstate);
  CK(cudaGetLastError());
  CK(cudaMemcpyAsync(out, b->d_wstate, sizeof(float) * WALL_STATE_LEN, cudaMemcpyDeviceToHost, b->last_stream));
  CK(cudaStreamSynchronize(b->last_stream));
  return SMG_OK;
}

int smg_snapshot(smg_batch* b, int32_t* map_off, smg_snap_object* objs, int cap_objs, int64_t* point_off, uint8_t* points,
                 int64_t cap_points, int64_t* n_points) {
  if (!b || !map_off || cap_objs < 0 || cap_points < 0) return fail(SMG_ERR_ARGS, "smg_snapshot: bad arguments");
  if (int r = sync_b(b)) return r;
  const Batch& B = b->B;
  const size_t MO = (size_t)B.M * B.O;
  if (!b->d_snap_rec) {
    if (int r = dalloc(b, &b->d_snap_rec, MO)) return r;
    if (int r = dalloc(b, &b->d_snap_out, MO)) return r;
    if (int r = dalloc(b, &b->d_snap_cnt, (size_t)B.M)) return r;
    if (int r = dalloc(b, &b->d_snap_src, MO)) return r;
    if (int r = dalloc(b, &b->d_snap_moff, (size_t)B.M + 1)) return r;
    if (int r = dalloc(b, &b->d_snap_npts, MO)) return r;
    if (int r = dalloc(b, &b->d_snap_poff, MO + 1)) return r;
  }
  cudaStream_t st = b->last_stream;
  k_snap_list<<<B.M, 256, 0, st>>>(B, b->d_snap_rec, b->d_snap_cnt, b->d_snap_npts, b->d_snap_src);
  k_snap_scan<<<1, SNAP_SCAN_THREADS, 0, st>>>(B, b->d_snap_cnt, b->d_snap_npts, b->d_snap_moff, b->d_snap_poff);
  CK(cudaGetLastError());
  CK(cudaMemcpyAsync(map_off, b->d_snap_moff, sizeof(int32_t) * (B.M + 1), cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  const int n = map_off[B.M];
  int64_t total = 0;
  CK(cudaMemcpy(&total, b->d_snap_poff + n, sizeof(int64_t), cudaMemcpyDeviceToHost));
  if (n_points) *n_points = total;
  const bool want_objs = objs && cap_objs >= n;
  const bool want_pts = points && cap_points >= total && total > 0;
  if (want_pts && (size_t)total * 15 > b->snap_pts_cap) {
    if (b->d_snap_pts) CK(cudaFree(b->d_snap_pts));
    b->d_snap_pts = nullptr;
    b->snap_pts_cap = 0;
    CK(cudaMalloc(&b->d_snap_pts, (size_t)total * 15));
    b->snap_pts_cap = (size_t)total * 15;
  }
  if ((want_objs || want_pts) && n > 0) {
    k_snap_pack<<<dim3(64, B.M), 256, 0, st>>>(B, b->d_snap_rec, b->d_snap_cnt, b->d_snap_src, b->d_snap_moff, b->d_snap_poff,
                                               want_objs ? b->d_snap_out : nullptr, want_pts ? b->d_snap_pts : nullptr);
    CK(cudaGetLastError());
    if (want_objs) {
      CK(cudaMemcpyAsync(objs, b->d_snap_out, sizeof(smg_snap_object) * n, cudaMemcpyDeviceToHost, st));
      if (point_off) CK(cudaMemcpyAsync(point_off, b->d_snap_poff, sizeof(int64_t) * (n + 1), cudaMemcpyDeviceToHost, st));
    }
    if (want_pts) CK(cudaMemcpyAsync(points, b->d_snap_pts, (size_t)total * 15, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
  } else if (want_objs && point_off) {
    point_off[0] = 0;
  }
  return n;
}

int smg_ply_header(int64_t n, char* out, int cap) {
  if (n < 0 || cap < 0) return fail(SMG_ERR_ARGS, "smg_ply_header: bad arguments");
  const std::string h = "ply\nformat binary_little_endian 1.0\nelement vertex " + std::to_string(n) +
                        "\nproperty float x\nproperty float y\nproperty float z\nproperty uchar red\nproperty uchar green\n"
                        "property uchar blue\nend_header\n";
  if (out && cap >= (int)h.size()) memcpy(out, h.data(), h.size());
  return (int)h.size();
}

int smg_set_reencode(smg_batch* b, int on) {
  if (!b) return fail(SMG_ERR_ARGS, "smg_set_reencode: bad arguments");
  if (int r = sync_b(b)) return r;
  b->B.reenc_on = on != 0;
  return SMG_OK;
}

int smg_get_work(smg_batch* b, int64_t* out, int n) {
  if (!b || !out || n <= 0) return fail(SMG_ERR_ARGS, "smg_get_work: bad arguments");
  if (int r = sync_b(b)) return r;
  std::vector<MapRec> maps((size_t)b->B.M);
  CK(cudaMemcpy(maps.data(), b->B.maps, sizeof(MapRec) * maps.size(), cudaMemcpyDeviceToHost));
  for (int k = 0; k < n; ++k) {
    out[k] = 0;
    if (k < SMG_WORK_N)
      for (const MapRec& r : maps) out[k] += r.wk[k];
    if (k == SMG_WK_H2D) out[k] += b->h2d_host;
  }
  return SMG_WORK_N;
}

}  // extern "C"
