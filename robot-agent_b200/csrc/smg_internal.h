// Internal device-state layout of an smg_batch (host + device visible PODs).
//
// HBM layout (one batch = M maps, O object slots per map, D embedding width):
//   MapRec[M]                 per-map scalars (ids, camera history, ceiling estimate, ApStats,
//                             insert-policy state, error word)
//   ObjRec[M*O]               per-object scalars of MapObject + ApState (scenemap objmap.hpp:157-187,
//                             objprob.hpp:156-193); objects are kept in the reference's list order
//                             through order[M*O] (slot indices), slots are recycled through a free list
//   rfrag[M*O*D]  f32         ApState::r_frag
//   views[M*O*(topk+1)*D] u16 ApState::views[].z (fp16 bits), one spare slot for insertion
//   cloud pool, C slots per map, one held by each object (ObjCloud, cloud.hpp:165-189):
//     cpts[cap] float4 (x,y,z relative to org, seq bits), crgb[cap] u32,
//     chkey/chidx[HC]   voxel-key -> point index hash (VoxelIndex, cloud.cpp:48-64),
//     ckey/cgen[HC]     4 cm contact-cell set (ApContactIdx, objprob.cpp:470-487), generation-cleared
//   per-frame scratch per (map, detection): back-projected points, observation records, cloud candidates
//   occupancy grid per map: hot (L, c8, flags, stamp) + cold sums, fixed window (OccGrid, grid.hpp:63-98)
//   view-first hash per map (ObjectMap::view_first_, objmap.hpp:333)
#pragma once
#include <stdint.h>

#include "../../include/smg.h"

#define SMG_MAX_DET 64
#define RE_CAND SMG_MAX_DET   // re-encode candidates per keyframe: objects seen this keyframe (<= detections)
#define SMG_TOPK_MAX 8
#define SMG_CAMS 32
#define SMG_CEIL_OBS 400
#define SMG_VIEW_BANDS 5
#define SMG_SUB 2048          // kPctMax (scenemap objmap.cpp:36)
#define SMG_MAX_EVENTS 1024   // per map per frame
#define VIEW_PIX (SMG_VIEW_MAX_SIDE * SMG_VIEW_MAX_SIDE)   // pixels of one best-view image slot
#define SMG_BINS_MAX 1440
#define SMG_MATCH_CELLS 12288 // kH * 3 / 4 (scenemap scan.cpp:319, :399)
#define WORK_SLOTS 16         // per-map work areas (cloud add CTAs per map)
#define CB_WORDS 16384        // contact bitset budget per cloud (words of 32 cells)

// error word bits
#define SMG_E_CAP_OBJ 1
#define SMG_E_CAP_PTS 2
#define SMG_E_CAP_GRID 4
#define SMG_E_CAP_VIEW 8
#define SMG_E_CAP_EVENTS 16
#define SMG_E_ARGS 32
#define SMG_E_CAP_REENC 64   // more re-encode candidates in a keyframe than RE_CAND
#define SMG_E_TRIM 128       // a cloud trim's selection ran past its depth limit (point order then differs)
#define SMG_E_CAP_WALLS 256  // wall extraction ran past a capacity (segments, runs of a row, lines, samples)

// Text model on the device (ApText, scenemap objprob.hpp:40-54, plus the class-kind table of
// ObjectMap::setClassKinds and the label tables the reference glue derives from label names).
struct TextDev {
  int dim, n_labels, rows;
  const float* text;         // rows x dim
  const int32_t* row_label;  // rows
  float scale, bias;
  const float* log_prior;    // n_labels or null
  const float* ls_mu;        // n_labels or null (with ls_sd)
  const float* ls_sd;
  const int32_t* parent;     // n_labels or null
  int object_label;
  const uint8_t* kinds;      // n_labels: 0 object, 1 structure, 2 static, 3 structural object (or null)
  const uint8_t* so_shape;   // n_labels: 1 door / window, 2 stairs / railing, 3 pillar (or null)
  const uint8_t* flat_ok;    // n_labels: wall-mounted flat object (or null)
};
#define KIND_OBJECT 0
#define KIND_STRUCTURE 1
#define KIND_STATIC 2
#define KIND_STRUCT_OBJ 3

// Per (map, frame) input descriptor on the device (smg_frame + host-derived scalars).
typedef struct {
  double stamp;
  int32_t w, h;
  const float* depth;
  const uint16_t* label;
  // host inputs the device reads in place (pinned, device-accessible), or null: the staging
  // images then hold only the pixels the chain reads, gathered by k_gather
  const float* depth_host;
  const uint16_t* label_host;
  float fx, fy, cx, cy;
  double T_mc[12];
  float T_bc[12];
  double base[3];
  double eef[2][3];
  float eef_base[2][3];
  int32_t n_det;
  uint16_t det_label[SMG_MAX_DET];
  float box[SMG_MAX_DET][4];
  int32_t cls[SMG_MAX_DET];
  float score[SMG_MAX_DET];
  const void* emb;
  int32_t emb_dtype;
  // host-derived with the host libm (same values the reference computes)
  double cam_w;          // camera optical-axis angular speed (objmap.cpp:520-530)
  int32_t cam_steady;    // cam_w <= move_max_cam_w
  double blur_fac;       // exp(-cam_w/blur_w) factor of viewKappa (1 when blur_w == 0)
  double cos_th, sin_th; // cos/sin of base yaw (grid.cpp:202)
  int32_t active;        // map takes part in this push
  // ObjectMap::updateHands (objmap.cpp:435-506): the per-hand gripper state machine depends only
  // on the gripper values and stamps, so the host runs it (host doubles, like the reference)
  // and passes per hand: act bit 0 = try a grasp, bit 1 = release (closed to the end after a
  // grasp), bit 2 = release (opened); gap = gripGap(grip) (objmap.cpp:387-397)
  int32_t hand_act[2];
  double hand_gap[2];
  int32_t hands_on;      // run the hand step (some map of the batch has used a gripper)
  // detector masks (sm_detections): bit masks on their own grid (mask_bits != null) or the label
  // image; the detector image size and its scale to the depth grid, as the reference computes
  // them (float in ObjectMap::update, objmap.cpp:635-636; double in buildReencode, :1377)
  const uint16_t* depth_mm;    // millimetre source converted into depth before the chain, or null
  const uint32_t* mask_bits;   // n_det x mask_words
  int32_t mask_w, mask_h, mask_words;
  float mask_sx, mask_sy, mask_ox, mask_oy;
  int32_t img_w, img_h;
  float sxu_f, syv_f;
  double sxu_d, syv_d;
  // sm_image::rgba (w x h RGBA8), device copy, or null; views_on = an RGB source the reference
  // uses: rgba present and the detector image the size of the depth image (capi.cpp:916)
  const uint8_t* rgba;
  int32_t views_on;
  // ObjFrame::wall_segs: wall_set = the keyframe carries a set (non-null pointer), which replaces
  // the map's stored one (Batch::wsegs, MapRec::n_wseg) before the chain; n_wseg segments at
  // wsegs (staging or the caller's device memory)
  const double* wsegs;
  int32_t n_wseg, wall_set;
} FrameDev;

// Observation (one detection after back-projection; scenemap objmap.cpp:52-74 `Obs`)
typedef struct {
  int32_t valid;         // 1 = survived to the structural test
  int32_t stage;         // where it stopped (diagnostics)
  int32_t det, sk, cls, trunc, n, nc, nsp;
  float score;
  double zmed, pos[3], ext[3], lo[3], hi[3], kappa;
  int32_t floor_drop;    // dropped by the 90th-percentile floor test (counts n_floor)
  // plane fit of the cloud candidates (apObsStructural, objmap.cpp:565-575)
  int32_t pl_ok;
  double pl_n[3], pl_thick, pl_inl, pl_zmed, pl_zlo, pl_zhi, pl_hspan;
  // association results
  int32_t obs_to, n_same, blocked, sec;
  // text model (apObsStructural, objmap.cpp:547-564): structure and structural-object
  // probabilities (ps = -1 without a text model or embedding), the single-fragment top label,
  // the most likely structural-object shape group, and the wall-like flags of the structural rules
  double ps, pso, top_p;
  int32_t top_lab, so_sh, wall_like, struct_look;
  // wall-line test of apObsStructural (objmap.cpp:606-611): of w_tot sampled candidates, w_near
  // lie within wall_d of a wall segment; through = the centre lies beyond a wall (:742-753)
  int32_t w_near, w_tot, through;
} ObsRec;

typedef struct __align__(16) {   // 16-byte aligned: staged in shared memory in 16-byte words
  uint32_t id;
  int32_t cls;
  double pos[3], ext[3], first_pos[3], lo[3], hi[3];
  uint32_t n_obs;
  double first_seen, last_seen;
  int32_t state, confirmed, moved, misses;
  double first_miss, miss_cam[3], last_miss_cam[3], last_miss_fwd[3];
  uint32_t n_vis_miss;
  double trk_pos[3], trk_t, trk_step[2];
  int32_t mv_cnt;
  double moving_t, move_from_t;
  float score;
  double last_kf, max_det_z, gone_t;
  int32_t appeared;
  int32_t cloud_slot;    // cloud pool slot owned by this object
  // ApState
  uint32_t ver;
  double k_frag;
  int32_t n_whole, n_views;
  int32_t view_slot[SMG_TOPK_MAX + 1];
  float vkappa[SMG_TOPK_MAX + 1];
  double vstamp[SMG_TOPK_MAX + 1];
  int32_t n_cams, cam_head;   // camera ring: n_cams newest, oldest at cams[cam_head]
  double cams[SMG_CAMS][7];
  int32_t n_wall_obs, n_ap_obs, n_struct_look;
  double whole_kappa;
  int32_t need_whole;
  double P[3];
  int32_t wall_like;
  uint32_t geo_ver;
  int32_t geo, drop, hide;
  double nrm_frag;       // |r_frag|^2 (ApState::nrm_frag, refreshed whenever r_frag changes)
  // whole-object views (ApState r_whole / k_whole / nrm_whole, objprob.hpp:158-169): has_whole = 1
  // once r_whole holds a vector (until a merge folds it into r_frag); vwhole[v] marks whole views
  double k_whole, nrm_whole;
  int32_t has_whole;
  int32_t vwhole[SMG_TOPK_MAX + 1];
  // hands (MapObject, objmap.hpp:175-178)
  int32_t held_by;       // hand holding it, -1 = none
  uint32_t parent;       // id of the object it rests on and follows, 0 = none
  double parent_rel[3], held_rel[3], grasp_pos[3];
  // best view (capi.cpp ViewSlot: the view's quality; has_view = a view is installed)
  double view_q;
  int32_t has_view;
  // label evidence and name (ApState lw_frag / lw_whole, post, name_*, top_*; the L_frag / L_whole
  // / post vectors live in Batch::lfrag / lwhole / post); has_post = post is not empty;
  // rename = apRename is due (seen this keyframe, merged, or a new whole view)
  double lw_frag, lw_whole;
  int32_t has_post, has_lfrag, has_lwhole, rename;
  int32_t name_lab, top_lab, rolled;
  float name_p, top_p, name_H;
  uint32_t post_ver;     // changes whenever post does (merge pair features read post)
  double gp_so;          // posterior mass of structure and structural-object labels (the guards' group)
  double maj, minr, hgt; // apStructObject shape of the cloud sample (5-95 % spans), with geo
  float vinl;            // inlier share of an upright dominant plane (ApState::vinl)
  float fw;              // share of the cloud sample within wall_d of a wall segment (ApState::fw)
} ObjRec;

typedef struct {
  double org[3];
  int32_t has_org;
  uint32_t version;
  int32_t n;
  uint32_t seq;
  double stamp;
  uint32_t vgen;         // generation of the voxel-key hash (clear = ++vgen)
  uint32_t cver;         // cloud version the contact index was built for
  // contact index (ApContactIdx): generation, count and cell range
  uint32_t cgen;
  int32_t cn;
  int64_t clo[3], chi[3];
  // dilated occupancy bitset of the contact cells over [clo-1, chi+1] (cb_ok = 1 when it fits)
  int32_t cb_ok, cb_dy, cb_dz, cb_wpr;
} CloudRec;

typedef struct {
  long long n_through, n_obs, n_wall, n_wall_name, n_ceil, n_floor, n_assoc, n_new, n_merge, n_obj_struct, n_reenc_req,
      n_reenc_done, n_blocked, n_wall_tall, n_so_big, n_bridge;
} StatsRec;

typedef struct {
  double t;
  uint32_t id;
  int32_t kind;
  uint32_t key;          // program-order key (phase << 24 | position)
  int32_t pad;
} EventRec;

// work counters, summed by smg_get_work: the per-unit terms of the algorithmic byte count
#define SMG_WK_OBS_PX 0      // pixels scanned by the per-detection back-projection (depth + label)
#define SMG_WK_DET 1         // detections processed
#define SMG_WK_VEC16 2       // memory vectors read by association, in units of D fp16 values
#define SMG_WK_UPD 3         // object vector updates (r_frag read + write, one view written)
#define SMG_WK_CLOUD 4       // cloud points written
#define SMG_WK_SCAN_PX 5     // depth pixels read by makeScan
#define SMG_WK_SCAN_PTS 6    // scan points inserted (match cells + laser hits + free rays)
#define SMG_WK_CELLS 7       // occupancy cells updated (one update per cell per scan)
#define SMG_WK_H2D 8         // host-input bytes the device read in place (pinned frames, k_gather)
#define SMG_WORK_N 9

// Merge-pass cache (the reference keeps one too, objmap.cpp:1137-1150): the embedding cosine and
// the contact fraction of an object pair depend only on the two objects' vectors (ver) and
// clouds (cloud version), so a pair whose four versions are unchanged reuses them.  Direct
// mapped; a collision only costs a recomputation.
#define PCACHE_SLOTS 8192
// one apAddView vector job of the keyframe (target object index tg of the frame's list)
struct UpdJob {
  int32_t tg, det, phys, zero;
  double k;
  double w;              // label weight k / kappa_ref (text model)
  int32_t lzero, ltext;  // L_frag starts from zeros; the job adds label evidence
};
struct PairCacheRec {
  uint32_t ida, idb, va, vb, ca, cb;
  double cs, contact;
};

typedef struct {
  uint32_t next_id;
  int32_t n_obj;
  int32_t n_free, n_cfree;
  int32_t n_evn;         // running event counter of the current phase
  int32_t err;
  double ceil_est;
  int32_t n_ceil;
  int32_t n_obs;         // observations surviving to association this frame
  int32_t n_events;
  int32_t n_pts;         // cloud-candidate lists emitted this frame
  int32_t n_targets;     // objects receiving cloud points / contact rebuilds this frame
  StatsRec st;
  double ceil_obs[SMG_CEIL_OBS];
  // Mapper2D insert policy (mapper2d.cpp:46-72)
  int32_t kf_first, kf_since, kf_last_changed, kf_inserted, kf_changed, kf_hits, kf_sig_n;
  double kf_last_ins[3];
  uint32_t scan_id;
  int32_t view_n;
  // cumulative work counters (algorithmic traffic of the path; see SMG_WK_*)
  long long wk[SMG_WORK_N];
  // whole-object re-encode requests of the last keyframe (k_reenc): count, candidate of each rank
  int32_t re_n, re_done;
  int32_t re_rank[RE_CAND];
  // best views (capi.cpp:903-998): version counter, views replaced by the last keyframe
  uint32_t view_ver;
  int32_t n_vnew;
  int32_t vnew[SMG_MAX_DET];   // candidate (detection) of each replaced view, install order
  int32_t n_wseg;        // the stored wall segments (ObjectMap::wsegs_), at Batch::wsegs
  int32_t wfr;           // segments this keyframe carries (ObjFrame::n_wall_segs; 0 = none)
  // wall extraction from the map's grid (sm_ctx wall state, capi.cpp:142-160): direction and the
  // stamps of its last measurement and of the last tilted extraction; has = segments extracted;
  // dirty = a visible grid value changed since; n_w segments at Batch::wall_w; the ignore
  // footprints of this keyframe (n_rect, changed = differ from the last extraction's)
  double w_th, w_th_t, w_full_t;
  int32_t w_has, w_dirty, n_w, n_rect, n_rect_prev, w_rchg;
} MapRec;

// Whole-object re-encode candidate of a keyframe (ReencReq, scenemap objmap.hpp:142-148, plus
// the ranking key); the mask bits live in Batch::reenc_bits, rows padded to whole words.
typedef struct {
  uint32_t id;
  int32_t ok;            // passed every test of buildReencode
  double prio;
  float kappa, box[4];
  double cam[6];
  int32_t mask_w, mask_h;
  int32_t win[4];        // rows r0..r1 and words w0..w1 written to the mask slot (zero elsewhere)
} ReencRec;

// Best-view candidate of a detection (BestView, bestview.hpp, plus the selection state): the
// images live at Batch::vrgb / vdepth / vmask, one fixed-size slot per (map, detection).
typedef struct {
  uint32_t id, version;
  int32_t cand;          // a candidate of this keyframe (quality test and crop geometry passed)
  int32_t final_;        // the view its object keeps after this keyframe
  double q, stamp;
  int32_t box[4], det_box[4];
  float mask_area, depth_m, score;
  double cam_T[12];
  int32_t w, h;
} ViewRec;

// ObjectMap::lastAssoc entry (DetAssoc, objmap.hpp:194-199)
typedef struct {
  uint32_t obj_id;
  int32_t n_valid;
  float area_px, depth_med;
} AssocRec;

// Per map per frame: emitted cloud-candidate list (ObsPoints, objmap.hpp:225-230)
typedef struct {
  uint32_t obj_id;
  int32_t det;
  int32_t n;
} PtsRec;

typedef struct {
  // sizes
  int32_t M, O, D, topk, cap, HC, HCC, pmax, max_det, W, H;
  int32_t C;                            // cloud slots per map (a pool shared by the map's objects)
  int32_t map0;                         // first map of the launch (maps are split into stream groups)
  int32_t reenc_on;                     // build whole-object re-encode requests (smg_set_reencode)
  int32_t work_n;                       // points per work area
  size_t work_stride;                   // bytes per work area
  int32_t gw_grid, gh_grid, gx0, gy0;   // occupancy window
  int32_t view_slots;                   // view-first hash slots per map
  int32_t scan_pmax;                    // makeScan grid capacity
  // parameters
  smg_params p;
  double cos_temper;                    // cos(temper_deg * pi / 180)  (objprob.cpp:317)
  double cos_gone_step;                 // cos(gone_step_deg * pi / 180) (objmap.cpp:1036)
  float inv_vox;                        // float(1.0 / max(1e-3, voxel)) (objmap.cpp:631)
  float inv_vox_cloud;                  // float(1.0 / voxel) (cloud.cpp:95)
  int16_t q_hit, q_miss, q_min, q_max;  // grid.cpp:110-113
  int32_t lut_off;
  // device arrays
  MapRec* maps;
  FrameDev* frames;
  ObjRec* objs;
  int32_t* order;        // [M*O]
  int32_t* freel;        // [M*O] free object-slot stack
  int32_t* cfreel;       // [M*C] free cloud-slot stack
  AssocRec* assoc;       // [M*max_det]
  float* rfrag;          // [M*O*D]
  float* mu;             // [M*O*D] ApState mu_c: float(r / |r|) of r_whole when k_whole > 0, else of r_frag
  float* rwhole;         // [M*O*D] ApState::r_whole
  uint16_t* views;       // [M*O*(topk+1)*D]
  CloudRec* clouds;      // [M*C]
  float4* cpts;          // [M*C*cap]
  uint32_t* crgb;        // [M*C*cap]
  uint64_t* chkey;       // [M*C*HC]
  uint32_t* chidx;       // [M*C*HC]
  uint32_t* chgen;       // [M*C*HC]
  uint32_t* cbits;       // [M*C*2*CB_WORDS] occupancy + dilated bitsets
  uint64_t* ckey;        // [M*C*HCC]
  uint32_t* cgen;        // [M*C*HCC]
  // per-frame scratch
  double* px;            // [M*max_det*pmax] x4 (X, Y, Z, ZC)
  int32_t* ppix;         // [M*max_det*pmax] x2 (PU, PV)
  double* pk;            // [M*max_det*pmax] x3 (kept X, Y, Z)
  float* cxyz;           // [M*max_det*pmax*3]
  int32_t* cpx;          // [M*max_det*pmax*2]
  double* sel;           // [M*max_det*pmax] x4 selection scratch
  ObsRec* obs;           // [M*max_det] by detection
  int32_t* obs_list;     // [M*max_det] detection index of observation a
  uint8_t* touched;      // [M*O]  by list position
  uint8_t* obj_hit;      // [M*O]
  double* gdot;          // [M*max_det*max_det] dot(z_b, z_a) of observations a < b (frame grouping)
  PtsRec* ptsl;          // [M*max_det]
  int32_t* tgt_slot;     // [M*O] cloud-addition targets (object slots)
  unsigned char* work;   // [M*WORK_SLOTS*work_stride]
  EventRec* events;      // [M*SMG_MAX_EVENTS]
  // merge pass scratch
  double* mcand_p;       // [M*O*8] candidate P
  uint32_t* mcand_ab;    // [M*O*8*2]
  uint32_t* mcand_key;   // [M*O*8] list positions i << 16 | j (the reference's enumeration order)
  int32_t* mcand_n;      // [M]
  int32_t* mgl;          // [M*MGL_CAP] gated merge pairs of the frame, i << 16 | j
  ReencRec* reenc;       // [M*RE_CAND]
  uint32_t* reenc_bits;  // [M*RE_CAND*re_words] closed masks, rows padded to whole words
  size_t re_words;       // H * ceil(W / 32)
  int32_t* mgl_n;        // [M] gated pairs; [M] next pair a warp takes (mgl_n + M)
  struct PairCacheRec* pcache;   // [M * PCACHE_SLOTS] merge-pass pair features of unchanged pairs
  double* sscr;          // [M * STRUCT_CTAS * STRUCT_SCR] k_struct scratch
  struct UpdJob* upd_job;  // [M * max_det] vector jobs of k_update, observation order
  // text model (smg_set_text_model)
  int32_t text_on;       // a text model with rows: label likelihoods and names run
  int32_t kinds_on;      // a class-kind table is set (isBig reads it)
  TextDev txt;
  float* lfrag;          // [M*O*C] ApState::L_frag
  float* lwhole;         // [M*O*C] ApState::L_whole
  float* post;           // [M*O*C] ApState::post
  float* llz;            // [M*max_det*C] apLabelLogLik of each detection's embedding
  double* wsegs;         // [M*SMG_WALL_SEGS_MAX*4] the stored wall segments of each map
  // wall extraction (smg_set_walls; allocated when first enabled)
  int32_t walls_on;
  int32_t wscr_side;     // side of the largest grid an extraction handles (the window rotated)
  uint64_t* wbits;       // [M*wbits_stride] occupancy bits: the window, then a rotated window
  size_t wbits_stride, wbits_half, wbits_cb;   // the rotated window at wbits_half, column bits at wbits_cb
  uint32_t* wruns;       // [M*wruns_stride] runs of rows, then of columns
  size_t wruns_stride;
  int32_t* wscr_i;       // [M*wscr_i_stride] ignore cell ranges (2*O int4), run counts
  size_t wscr_i_stride;
  double* wrect;         // [M*O*4] ignore footprints of the keyframe
  double* wrect_prev;    // [M*O*4] those of the last extraction
  double* wall_w;        // [M*SMG_WALL_SEGS_MAX*4] extracted segments (no bridges)
  double* wall_raw;      // [M*SMG_WALL_SEGS_MAX*4] raw segments of a rotated extraction
  double* wall_tmp;      // [M*SMG_WALL_SEGS_MAX*4] column segments while the rows' are chained
  unsigned char* wall_lines;   // [M*SMG_WALL_SEGS_MAX*16] refined lines of each raw rotated segment (32 bytes each)
  int32_t* wall_lcnt;    // [M*SMG_WALL_SEGS_MAX] their counts
  // best views (allocated on the first push with an RGB image)
  ViewRec* vrec;         // [M*max_det]
  uint8_t* vrgb;         // [M*max_det*VIEW_PIX*3]
  uint16_t* vdepth;      // [M*max_det*VIEW_PIX]
  uint8_t* vmask;        // [M*max_det*VIEW_PIX]
  int64_t* upd_tg;         // [M * max_det] target objects (global slot) of those jobs
  int32_t* upd_n;          // [M * 2] jobs, targets
  // view-first hash (markView)
  int64_t* vkey;         // [M*view_slots], INT64_MIN = empty
  double* vfirst;        // [M*view_slots*5]
  // RANSAC adaptive iteration table need[nsamp][cnt] (objprob.cpp:161), host libm
  int32_t* need_tab;     // [NEED_N*NEED_N]
  // occupancy grid
  int16_t* gL;           // [M*gw*gh]
  int8_t* gc8;
  uint8_t* gflags;
  uint32_t* gstamp;
  float4* gcold;         // sx, sy, nx, ny
  uint32_t* gcnt;        // cnt | cntn << 16
  unsigned long long* gtouch;   // per-scan first-touch key
  int8_t* lut8;          // export8 LUT (grid.cpp:118-123), host libm
  float* lutp;
  // makeScan scratch
  float4* sP;            // [M*scan_pmax] base-frame point + optical z
  int16_t* pbin;         // [M*scan_pmax]
  float* phs2;           // [M*scan_pmax]
  float* bin_cos;        // [bins] cos/sin of bin centres, host libm (scan.cpp:435-437)
  float* bin_sin;
  unsigned long long* hit_key;   // [M*bins] (rr2 bits << 32 | pixel)
  float* floor_r;        // [M*bins]
  int16_t* sig;          // [M*bins] this scan's signature
  int16_t* ins_sig;      // [M*bins] signature of the last inserted scan
  int64_t* mkey;         // [M*scan_pmax] match key per pixel (INT64_MIN = none)
  float4* mval;          // [M*scan_pmax] px, py, ux, uy
  int64_t* mh_key;       // [M*16384] match-cell hash
  int32_t* mh_first;     // [M*16384]
  int32_t* mh_cell;      // [M*16384] rank of the cell in first-seen order
  int32_t* mcell_first;  // [M*scan_pmax] first pixel of cell rank r
  int32_t* mcell_cnt;    // [M*scan_pmax]
  int32_t* mcell_off;    // [M*scan_pmax]
  int32_t* mcell_pix;    // [M*scan_pmax]
  float* sc_pts;         // [M*(2*bins + SMG_MATCH_CELLS)*6] insert point list: x, y, nx, ny (base frame)
  int32_t* sc_n;         // [M*3] nm, nh, nf
  int32_t* err_global;
} Batch;
