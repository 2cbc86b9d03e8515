/* smg.h — C ABI of the B200-native scenemap objprob per-frame update.
 *
 * One `smg_batch` holds M independent maps on one GPU: each map is one scenemap
 * (ObjectMap + Mapper2D occupancy grid).  A call to smg_push_frames runs, for every map,
 * the reference keyframe path for one depth frame:
 *   Mapper2D::keyframe  (scenemap src/mapper2d.cpp:27-87: makeScan + OccGrid::insert)
 *   ObjectMap::update   (scenemap src/objmap.cpp:516-1086)
 *   ObjectMap::addPoints for every emitted observation cloud (scenemap src/capi.cpp:986-992)
 * entirely on the device, on the caller's stream.  Nothing falls back to the CPU: without a
 * usable sm_100 device every entry point returns SMG_ERR_DEVICE.
 *
 * Conventions (scenemap include/scenemap.h:421 convention): 0 = ok, negative = error.
 * No exception crosses this ABI.  One host thread per batch; calls on one batch must not
 * overlap.  All pointers are plain; "device" pointers are CUDA device addresses.
 */
#ifndef SMG_H
#define SMG_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  SMG_OK = 0,
  SMG_ERR_ARGS = -1,       /* bad arguments / unsupported input form */
  SMG_ERR_PARAM = -2,      /* unknown parameter key */
  SMG_ERR_CAPACITY = -3,   /* an object / point / cell capacity would be exceeded */
  SMG_ERR_DEVICE = -4,     /* CUDA error, or the device error word was set */
  SMG_ERR_UNSUPPORTED = -5,/* a known reference input or parameter this build does not implement */
};

enum { SMG_MEM_DEVICE = 0, SMG_MEM_HOST = 1 };
/* wall segments a keyframe may carry (smg_frame::wall_segs) or an extraction may find */
#define SMG_WALL_SEGS_MAX 1024
/* the wall state vector (sm_snap_wall_state, scenemap include/scenemap.h:96-99) */
#define SMG_WALL_STATE_LEN 56
enum { SMG_EMB_F32 = 0, SMG_EMB_BF16 = 1 };

/* Parameters.  Field names and defaults mirror the reference structs:
 * ObjParams (scenemap include/scenemap/objmap.hpp:50-129), ApParams (objprob.hpp:56-142),
 * KappaParams (bestview.hpp:67-69), GridParams (grid.hpp:18-21), ScanParams (scan.hpp:37-48),
 * MapperParams (mapper2d.hpp:14-26).  Fill with smg_params_default, override with
 * smg_params_apply ("key=val,..." — the reference's applyParams key names, objmap.cpp:132-205). */
typedef struct smg_params {
  /* ObjParams */
  int32_t min_points;
  float zmin, zmax, hand_r, hand_frac;
  double big;
  int32_t confirm;
  double prune_s, moved_d;
  int32_t gone_misses;
  double gone_min_s, mad_k, mad_floor, grow_max, max_ext, occl;
  int32_t min_px;
  double self_pad;
  int32_t step, max_pts;
  double voxel;
  int32_t cloud_cap;
  double cloud_hand_r, body_r, merge_min_ext, floor_h;
  int32_t absent_samples;
  double absent_vis, absent_min_px, absent_det_k;
  int32_t gone_misses_big;
  double gone_min_s_big;
  int32_t spurious_obs;
  double gone_view_d, gone_step_d, gone_step_deg, gone_eps;
  double link_v, link_d0, link_max_d;
  int32_t link_min_obs;
  double link_wait_s, link_window_s, link_view_gap_s, view_cell;
  int32_t move_n;
  double move_v, move_min_d, move_max_cam_w;
  double ap_q_pos, ap_r0, ap_r1;
  /* ApParams */
  double same_p, merge_p, w[8], wm[8], guard_obj, guard_obs, name_veto;
  int32_t bridge_drop, frame_group;
  double cos0, gate, contact_cell;
  int32_t contact_samples, topk;
  double temper_d, temper_deg, temper, kappa_ref;
  double plane_thick, ransac_tau0, ransac_tau_k, ransac_tau_max, obj_tau, plane_inl, obj_plane_inl;
  int32_t ransac_iters;
  double wall_vert, ceil_z, horiz, floor_z, ceil_band, ceil_frac, ceil_wide;
  double tall_h, tall_floor, tall_ceil, tall_w, tall_ps, tall_w_any;
  double obj_wall_span, obj_wall_top, obj_wall_h, obj_thick;
  double struct_obj_p;
  int32_t struct_obj_min_views;
  double link_cos;
  /* KappaParams */
  double kap_k0, kap_s0, kap_trunc, kap_d0, kap_occ, kap_blur_w;
  /* GridParams + ScanParams + MapperParams (insert policy) */
  float grid_res, l_hit, l_miss, l_min, l_max;
  float scan_zmin, scan_zmax, band_lo, band_hi;
  int32_t bins;
  float self_r, eef_r, arm_r, shoulder[2][3], match_hi, vert_nz, match_cell;
  int32_t dense, change_bins, change_cells, still_every;
  /* ApParams re-encode requests (objprob.hpp:90-93) */
  int32_t reenc_max;
  double reenc_gain, reenc_min_vis;
  int32_t reenc_min_px;
  /* ObjParams hands (objmap.hpp:66-76): grasp radius, closed-gripper threshold, hands used,
   * grasp checks, gripper settling, and the gripper value -> finger gap table (ascending,
   * linear in between, clamped outside; n_grip_gap <= 8 pairs) */
  double grasp_r;
  float grip_closed;
  int32_t n_hands;
  double grasp_max_w, grasp_min_gap, grasp_w_tol, grip_settle_s, grip_settle_eps;
  int32_t n_grip_gap;
  double grip_gap[8][2];
  /* ApParams text-model rules (objprob.hpp:84-136): naming (name_tau, name_wmax, size_w,
   * whole_w, geo_w), the structure guards of association and merging (struct_look_block,
   * flat_max_w), the small-wall-plane rules (wall_big, struct_p) and the structural-object
   * size checks (so_*, wallhug_*, big_vinl).  They act only with a text model
   * (smg_set_text_model). */
  double name_tau, name_wmax, size_w, whole_w, geo_w, flat_max_w, wall_big, struct_p;
  double so_dw_w, so_dw_thick, so_max_h, so_pillar, so_stairs, so_dw_min, so_hide_k, wallhug_frac, wallhug_w, big_vinl;
  int32_t struct_look_block, so_min_obs;
  /* ApParams wall-line rules (objprob.hpp:101-117): a point within wall_d of a wall segment is
   * on a wall line, wall_frac of a thin upright fragment's points on one makes it a wall plane;
   * a fragment whose centre lies beyond a wall segment, seen from the camera, by more than
   * through_d is dropped; an object whose dominant plane is thinner than obj_flat_thick with
   * obj_flat_frac of its points within obj_flat_d of a wall line is a flat plane on the wall
   * (geo 3), dropped unless its flat-object and structural-object names hold flat_keep_p.
   * bridge_max: the longest gap between two collinear segments that the extracted set closes
   * (capi.cpp:873-887; 0 = none).  They act when a keyframe carries wall segments. */
  double wall_d, wall_frac, through_d, bridge_max, obj_flat_thick, obj_flat_d, obj_flat_frac, flat_keep_p;
} smg_params;

/* One frame of one map.  depth/label/emb/dets/masks live in device memory (SMG_MEM_DEVICE) or
 * in host memory (SMG_MEM_HOST: copied in by the call, on the caller's stream).
 * Detections come in one of two forms: a label image (the mask of detection k is the set of
 * pixels whose label equals det_label[k]: a mask grid equal to the depth grid), or the
 * reference's bit masks on their own grid (mask_bits below). */
typedef struct smg_frame {
  double stamp;
  int32_t w, h;
  const float* depth;          /* w*h optical depth, metres */
  const uint16_t* label;       /* w*h instance labels */
  float fx, fy, cx, cy;
  double T_mc[12];             /* map <- camera optical, row-major 3x4 (ObjFrame::T_mc) */
  float T_bc[12];              /* base <- camera optical (DepthView::T_bc) */
  double base[3];              /* base pose in the map (x, y, yaw): the grid insert pose */
  double eef[2][3];            /* hand points, map frame (ObjFrame::eef) */
  float eef_base[2][3];        /* hand points, base frame (BodyState::eef) */
  int32_t n_det;
  const uint16_t* det_label;   /* n_det */
  const float* box;            /* n_det x 4: x0 y0 x1 y1 pixels */
  const int32_t* cls;          /* n_det */
  const float* score;          /* n_det or NULL */
  const void* emb;             /* n_det x emb_dim, L2-normalised */
  int32_t emb_dtype;           /* SMG_EMB_F32 | SMG_EMB_BF16 */
  float grip[2];               /* gripper values (ObjFrame::grip, rad; the reference's default is
                                  1 = open: a zero-filled frame means a closed gripper) */
  /* The detector's masks in the reference's own form (sm_detections, scenemap
   * include/scenemap.h:20-34), used instead of label/det_label when mask_bits is set:
   * n_det x ceil(mask_w * mask_h / 32) words, cell (i, j) is bit j * mask_w + i, LSB first;
   * cell (i, j) covers detector-image x in [i sx + ox, (i+1) sx + ox), y likewise.  img_w x img_h
   * is the detector image (box is in its pixels); 0 means the depth image's size.  The mask grid
   * may be at most max_w x max_h cells. */
  const uint32_t* mask_bits;
  int32_t mask_w, mask_h;
  float mask_sx, mask_sy, mask_ox, mask_oy;
  int32_t img_w, img_h;
  /* ObjFrame::depth_mm: depth as uint16 millimetres (read as mm * 1e-3f, like the reference),
   * used when depth is NULL */
  const uint16_t* depth_mm;
  /* sm_image::rgba: w*h RGBA8 colour image registered with the depth image, or NULL.  With it
   * (and a detector image the size of the depth image), the keyframe also colours the cloud
   * points it adds (gatherRgbHost, bestview.cpp) and picks best views (capi.cpp:903-998):
   * smg_get_views.  Without it, points are grey (128) and no view is picked, as in the
   * reference with no RGB source. */
  const uint8_t* rgba;
  /* ObjFrame::wall_segs / n_wall_segs (objmap.hpp:219-220): n_wall_segs x (ax, ay, bx, by),
   * map metres, at most SMG_WALL_SEGS_MAX, or NULL; in the memory the push's `where` names (like
   * depth).  A non-NULL set replaces the map's stored
   * one (ObjectMap::wsegs_, read by apStructObject) and this keyframe's fragments get the
   * wall-line tests (apObsStructural, the see-through drop); NULL keeps the stored set and
   * skips the keyframe's tests, as in the reference (objmap.cpp:534, 605, 742). */
  const double* wall_segs;
  int32_t n_wall_segs;
} smg_frame;

typedef struct smg_batch smg_batch;

/* sizeof(smg_params), for bindings that treat the struct as an opaque buffer. */
int smg_params_size(void);
/* scenemap objmap.hpp:50-129 defaults (+ objprob.hpp:56-142, bestview.hpp:67-69, grid.hpp:18-21,
 * scan.hpp:37-48, mapper2d.hpp:14-26). */
int smg_params_default(smg_params* p);
/* ObjectMap::applyParams (scenemap src/objmap.cpp:132-205): "key=val,...".  Returns the number
 * of unknown keys (0 = all known), or SMG_ERR_ARGS.  Keys of reference features this build does
 * not run (the inspect pass and the export filter: inspect, ap_export_named) are accepted at
 * their reference default only; any other value makes the call return SMG_ERR_UNSUPPORTED (all
 * other keys are still applied) and smg_last_error names them. */
int smg_params_apply(smg_params* p, const char* kv);

/* ObjectMap::setCloudParams (scenemap objmap.hpp:255-258): voxel > 0 and cap > 0 override. */
int smg_params_set_cloud(smg_params* p, double voxel, int cap);

/* Create M maps on device `dev`.  max_objects: object slots per map; emb_dim: embedding width
 * (<= 2048); max_w/max_h: largest frame; max_det: detections per frame (<= 64);
 * grid_w/grid_h and grid_x0/grid_y0: the fixed occupancy window in global cell indices.
 * Replaces `new ObjectMap(p)` + `Mapper2D(p)` (scenemap objmap.hpp:235, mapper2d.hpp:39). */
int smg_create(const smg_params* p, int n_maps, int max_objects, int emb_dim, int max_w, int max_h, int max_det, int grid_w,
               int grid_h, int grid_x0, int grid_y0, int dev, smg_batch** out);
/* smg_create with the object clouds in a pool of max_clouds slots per map (<= max_objects).  An
 * object slot holds the object's scalars and vectors (about 28 KB at D = 1152); a cloud slot
 * reserves a full-capacity cloud with its voxel index and contact cells (about 1.2 MB at
 * cloud_cap 8000), and every live object holds one.  A map whose live objects would exceed
 * max_clouds sets the capacity bit of its error word (the observation that would have created
 * the object is dropped), as running out of object slots does.  smg_create is this call with
 * max_clouds = max_objects. */
int smg_create_pooled(const smg_params* p, int n_maps, int max_objects, int max_clouds, int emb_dim, int max_w, int max_h,
                      int max_det, int grid_w, int grid_h, int grid_x0, int grid_y0, int dev, smg_batch** out);
int smg_destroy(smg_batch* b);

/* One keyframe for each of the first n maps (frames[i] -> map i).  Replaces, per map,
 * the keyframe block of sm_push_image_rgb (scenemap src/capi.cpp:811-992):
 * Mapper2D::keyframe, ObjectMap::update, ObjectMap::addPoints, and on frames that carry
 * detection embeddings ObjectMap::buildReencode (capi.cpp:1002-1010).  `stream` is a cudaStream_t
 * (NULL = the legacy default stream).  Returns before the device work finishes; results
 * are read with the getters below (which synchronise the stream). */
int smg_push_frames(smg_batch* b, const smg_frame* frames, int n, int where, void* stream);

/* Whether pushes build the whole-object re-encode requests (on by default).  The reference's
 * push builds them on every frame that carries detection embeddings (capi.cpp:1002-1010); a
 * caller that never encodes whole-object crops can switch the stage off.  With it off,
 * smg_get_reencode returns no requests. */
int smg_set_reencode(smg_batch* b, int on);

/* ApText (scenemap objprob.hpp:40-54), device pointers (host pointers for smg_set_text_model): rows x dim L2-normalised text
 * embeddings, the label of each row, SigLIP logit scale/bias, and the optional per-label
 * log prior, log-size Gaussian (mu, sd; sd <= 0 = unused) and hypernym parent (-1 = none). */
typedef struct smg_text {
  int32_t dim, n_labels, rows;
  const float* text;
  const int32_t* row_label;
  float scale, bias;
  const float* log_prior;
  const float* ls_mu;
  const float* ls_sd;
  const int32_t* parent;
  int32_t object_label;
} smg_text;
/* The text model of every map of the batch (ObjectMap::setTextModel and setClassKinds; the
 * reference sets them through sm_set_labels, sm_set_text_model and sm_set_label_stats,
 * scenemap.h:396-401, capi.cpp:1769-1806).  With it, each observation's label likelihood
 * (apLabelLogLik) gives its structure probabilities for the structural rules and the
 * association guards (objmap.cpp:547-622, :785-800), every view adds to the object's label
 * evidence (apAddView), and objects seen in a keyframe, merged objects and objects with a new
 * whole view are renamed (apRename -> apName: posterior, name, class), which the merge pass,
 * the structural-object test and isBig then read.  t: the text rows and label statistics
 * (host arrays, copied; rows may be 0 for class kinds alone); per label, host arrays of
 * t->n_labels bytes (NULL = all 0): kinds (0 object, 1 structure, 2 static, 3 structural
 * object: door / window / stairs / pillar), so_shape (1 door or window, 2 stairs or railing,
 * 3 pillar, 0 other: what capi.cpp:1778-1784 derives from the label names) and flat_ok
 * (wall-mounted flat objects: picture, TV, clock ..., capi.cpp:1774-1777).  Call it before the
 * first push; n_labels <= 1024 and dim = the batch's emb_dim when rows > 0. */
int smg_set_text_model(smg_batch* b, const smg_text* t, const uint8_t* kinds, const uint8_t* so_shape, const uint8_t* flat_ok);
/* The name state of object i of map m (ApState after apName): post (n_labels floats, zeros when
 * the object has none yet), lab3 = {name_lab, top_lab, rolled}, val3 = {name_p, top_p, name_H};
 * returns n_labels when the object has a posterior, else 0. */
int smg_get_object_name(smg_batch* b, int m, int i, float* post, int32_t* lab3, float* val3);

/* ---- results (device -> host on request; each getter synchronises the batch stream) ---- */
/* A best view (scenemap include/scenemap/bestview.hpp BestView; chosen as capi.cpp:903-998
 * does: quality q = valid mask area x score, a detection's crop replaces the object's view when
 * q >= the view's q (ties: the newer), moved / put-down events reset the view's q to 0).  box:
 * the crop (detection box + 10 % per side, clipped), det_box: the rounded detection box, both
 * in image pixels [x0, y0, x1, y1); w x h: the crop's size (longer side <= 256). */
/* sm_object (scenemap include/scenemap.h:55-66) of an exportable object as sm_snapshot lists it
 * (capi.cpp:1051-1067), plus what scene.json and sm_snap_movable / sm_snap_points read of it. */
typedef struct smg_snap_object {
  uint32_t id;
  int32_t name_lab;            /* class label (sm_object::name is that label's name); -1 = "?" */
  float score;
  double pos[3], extent[3], first_pos[3];   /* map */
  uint32_t n_obs;
  double last_seen;
  int32_t state;               /* SM_SEEN 0, SM_GONE 1, SM_MOVED 2, SM_HELD 3 (held by a hand) */
  int32_t structural;          /* static or structural-object kind, or a side longer than big */
  int32_t movable;             /* neither static nor structural-object kind (sm_snap_movable) */
  int32_t n_points;            /* cloud points (sm_snap_points) */
  double cloud_stamp;          /* stamp of the cloud's last addition */
} smg_snap_object;

typedef struct smg_view {
  uint32_t id, version;
  double q, stamp;
  int32_t box[4], det_box[4];
  float mask_area, depth_m, score;
  double cam_T[12];
  int32_t w, h;
} smg_view;
#define SMG_VIEW_MAX_SIDE 256
typedef struct smg_object {
  uint32_t id;
  int32_t cls;
  double pos[3], ext[3], first_pos[3], lo[3], hi[3];
  uint32_t n_obs;
  double first_seen, last_seen;
  int32_t state, confirmed, moved, misses;
  uint32_t n_vis_miss;
  float score;
  double max_det_z, last_kf;
  int32_t appeared;
  int32_t cloud_n;
  uint32_t cloud_version;
  double cloud_org[3];
  uint32_t ap_ver;
  double k_frag;
  int32_t n_views, n_ap_obs, need_whole;
  double P[3];
  int32_t n_cams, geo;
  double k_whole;              /* ApState::k_whole (sum of whole-view kappas) */
  int32_t n_whole;             /* whole views since the last merge (ApState::n_whole) */
  int32_t held_by;             /* hand holding the object, -1 = none (MapObject::held_by) */
  uint32_t parent;             /* object it rests on / in and follows, 0 = none (MapObject::parent) */
  double parent_rel[3];
  /* ApState wall-line state: wall_like (a thin upright plane on a wall line or structure-looking),
   * hide (apStructObject: kept but not exported as a node), n_wall_obs (wall-like fragments
   * seen), fw (share of the cloud sample within wall_d of a wall segment) */
  int32_t wall_like, hide, n_wall_obs;
  float fw;
} smg_object;

/* ObjectMap::objects() (scenemap objmap.hpp:242) of map m, in the reference's order. */
int smg_get_objects(smg_batch* b, int m, smg_object* out, int cap);
/* r_frag (emb_dim floats) and the top-k views (fp16 bits, emb_dim each) of object i of map m. */
int smg_get_object_vectors(smg_batch* b, int m, int i, float* r_frag, uint16_t* views, float* vkappa, double* vstamp, int vcap);
/* Cloud of object i of map m: points relative to cloud_org (float xyz) and seq; returns count. */
int smg_get_object_cloud(smg_batch* b, int m, int i, float* xyz, uint32_t* seq, int cap);
/* Cloud colours of object i of map m (ObjCloud point r, g, b; grey without an RGB source),
 * 3 bytes per point in the order of smg_get_object_cloud; returns count. */
int smg_get_object_cloud_rgb(smg_batch* b, int m, int i, uint8_t* rgb, int cap);
/* The views of map m that its last keyframe replaced, in the order the reference installs
 * them (its views map keeps, per object id, only the last).  Images (may be NULL) are written
 * at a fixed stride per view, row-major and packed to w x h: rgb at rgb + v * 256*256*3 (area
 * average of the crop box), depth at depth + v * 256*256 (uint16 mm, nearest, 0 = none;
 * cropDepthMm) and mask at mask + v * 256*256 (255 inside the detection mask; cropMask).  They
 * are valid until the next push.  Returns the number of views (up to cap copied). */
int smg_get_views(smg_batch* b, int m, smg_view* out, uint8_t* rgb, uint16_t* depth, uint8_t* mask, int cap);
/* ObjectMap::lastAssoc() (objmap.hpp:251) of map m: per detection obj_id, n_valid, area_px, depth_med. */
int smg_get_assoc(smg_batch* b, int m, uint32_t* obj_id, int32_t* n_valid, float* area_px, float* depth_med, int cap);
/* ApStats (objmap.hpp:132-139) of map m, 16 counters in declaration order. */
int smg_get_stats(smg_batch* b, int m, int64_t* out16);
/* Events of the last frame of map m (ObjEvent, objmap.hpp:150-155): t, id, kind. */
int smg_get_events(smg_batch* b, int m, double* t, uint32_t* id, int32_t* kind, int cap);
/* Occupancy window of map m: log-odds (1/256 fixed point), seen flag, export8 value
 * (OccGrid::export8, grid.cpp:209-213), grid_w*grid_h cells, row-major. */
int smg_get_grid(smg_batch* b, int m, int16_t* L, uint8_t* seen, int8_t* c8);
/* Keyframe stats of the last frame of map m: inserted, changed_cells, n_hits (KeyframeStats). */
int smg_get_keyframe(smg_batch* b, int m, int32_t* out3);
/* Association of all maps in one read: obj_id[m * max_det + k] (0 = no object). */
int smg_get_assoc_all(smg_batch* b, uint32_t* obj_id);
/* The same read without waiting, for callers that keep pushes in flight: enqueued on the stream of
 * the last push, after its keyframe; obj_id should be pinned host memory (the copy is then
 * asynchronous) and stays the caller's until smg_wait_read(b, *ticket) returns.  At most four
 * reads are in flight (a fifth waits for the oldest). */
int smg_get_assoc_all_async(smg_batch* b, uint32_t* obj_id, int64_t* ticket);
int smg_wait_read(smg_batch* b, int64_t ticket);
/* Whole-object re-encode request (sm_reenc_req, scenemap include/scenemap.h:407, plus the
 * request's camera and mask grid; ReencReq, objmap.hpp:142-148): object id, crop box in image
 * pixels (x0 y0 x1 y1), the view kappa the whole view will carry, the camera position and
 * optical axis (map frame) at request time, and the mask grid (= the frame's image grid). */
typedef struct smg_reenc_req {
  uint32_t id;
  float box[4];
  float kappa;
  double cam[6];
  int32_t mask_w, mask_h;
} smg_reenc_req;
/* Re-encode requests of map m from its last keyframe (sm_reencode_requests, scenemap.h:408),
 * best first.  bits (may be NULL) receives the projected mask of request r at
 * bits + r * ceil(max_w * max_h / 32): ceil(mask_w * mask_h / 32) words, bit q = pixel q of
 * the row-major mask grid, LSB first.  Returns the number of requests (up to cap copied). */
int smg_get_reencode(smg_batch* b, int m, smg_reenc_req* reqs, uint32_t* bits, int cap);
/* The whole-object embeddings the caller computed for the re-encode requests (sm_set_object_
 * embeddings, scenemap include/scenemap.h:410, capi.cpp:1825-1835): entry i is an L2-normalised
 * fp32 embedding (dim = the batch's emb_dim) of object ids[i] of map maps[i].  It is added as a
 * whole view (ObjectMap::addWholeView, objmap.cpp:1361-1369: r_whole, whole-first view order,
 * need_whole cleared) when that map's last keyframe requested the object and the object still
 * exists, with the request's kappa and camera; otherwise it is ignored, as in the reference.
 * Entries of one map apply in call order.  n <= n_maps * 64.  Runs on `stream` after the last
 * push; with SMG_MEM_HOST arrays the call returns when they have been read. */
int smg_set_object_embeddings(smg_batch* b, const int32_t* maps, const uint32_t* ids, const float* emb, int n, int dim, int where,
                              void* stream);
/* r_whole (emb_dim floats, zeros when the object has none) and k_whole of object i of map m;
 * returns n_whole. */
int smg_get_object_whole(smg_batch* b, int m, int i, float* r_whole, double* k_whole);

/* Wall extraction from each map's own occupancy grid before every object update, as the
 * reference's image push does (sm_push_image: refreshWalls, scenemap src/capi.cpp:646-698, and the
 * bridged list of :866-890 handed to ObjectMap::update as ObjFrame::wall_segs; walls.cpp).  The
 * floor footprints of confirmed, named objects are ignored; the dominant wall direction is
 * re-measured at most every 2 s of frame stamps; tilted maps are extracted along it (at most
 * every 0.5 s); the keyframe then carries the segments plus the bridges of gaps up to
 * ap_bridge_max between collinear ones.  on = 1 enables (and resets the extraction state), 0
 * disables; with it on, frames must not carry their own wall_segs.  The extraction runs on the
 * batch's grid window (the reference runs it on its grown grid). */
int smg_set_walls(smg_batch* b, int on);
/* sm_snap_wall_segments (scenemap include/scenemap.h:100, capi.cpp:1247-1257): the segments of
 * map m's last extraction (n x ax ay bx by, map metres, no bridges); returns their count (may
 * exceed cap), or -1 when walls are off or not yet extracted. */
int smg_get_wall_segments(smg_batch* b, int m, double* out, int cap);
/* sm_snap_wall_state (scenemap include/scenemap.h:96-99, capi.cpp:1239-1245; walls.hpp: the first
 * occupied cell along 16 rays from the pose, then the 8 nearest segments in the robot frame) of
 * map m at pose (x, y, yaw): SMG_WALL_STATE_LEN floats.  Returns -1 when walls are off or not yet
 * extracted.  Segments at equal distance come in segment order (the reference's partial_sort
 * leaves their order unspecified). */
int smg_wall_state(smg_batch* b, int m, const double pose[3], float* out);

/* The object-memory snapshot of every map in one call: sm_snapshot's object list (scenemap
 * capi.cpp:1051-1067: ObjectMap::exportable objects in object order, the hand's objects as
 * SM_HELD) and dsg_save's object point files (dsg_save.cpp:70-89 plyBytes: per point float x, y,
 * z in map metres and uchar r, g, b, 15 bytes, little-endian), packed on the device.
 * map_off (n_maps + 1 entries): map m's objects are [map_off[m], map_off[m+1]).  Returns the
 * number of objects n.  objs (and point_off, n + 1 entries: object i's points are records
 * [point_off[i], point_off[i+1])) are filled when cap_objs >= n; points when cap_points >= the
 * total records, which *n_points receives.  Call once with NULL buffers to size them. */
int smg_snapshot(smg_batch* b, int32_t* map_off, smg_snap_object* objs, int cap_objs, int64_t* point_off, uint8_t* points,
                 int64_t cap_points, int64_t* n_points);
/* The PLY header plyBytes writes before n vertex records (ASCII, binary_little_endian 1.0, x y z
 * float, red green blue uchar); returns its length, or the needed size when cap is too small. */
int smg_ply_header(int64_t n, char* out, int cap);

/* Per-kernel device time with CUDA events on the launch stream (instrumentation, off by
 * default).  smg_timing_read fills ms[k] (total milliseconds) and n[k] (launches) for the
 * SMG_NUM_KERNELS kernels of the keyframe chain and resets the counters; names[k] is static. */
#define SMG_NUM_KERNELS 18
int smg_timing_enable(smg_batch* b, int on);
int smg_timing_read(smg_batch* b, double* ms, int64_t* n, const char** names);
/* First failed self-check of a -DSMG_CHECKS build: (site, index, bound); all zero when none
 * (always zero in the production build). */
int smg_debug_check(smg_batch* b, uint64_t* out3);
/* Instrumentation builds (-DSMG_PHASE_TIMING) only: per-phase clock cycles of the chain's
 * largest kernels (thread 0 of every block), out[2k] cycles and out[2k+1] marks for k < 64,
 * then reset.  The production build returns SMG_ERR_UNSUPPORTED. */
int smg_phase_read(uint64_t* out);
/* Device error word (0 = none) and a static description of the last host-side error. */
int smg_error_word(smg_batch* b);
const char* smg_last_error(void);
/* Number of kernels the library has launched since creation (instrumentation). */
int64_t smg_kernel_launches(smg_batch* b);
/* Cumulative work counters summed over the maps of the batch (instrumentation, no reference
 * counterpart): out[0] pixels scanned by the detection back-projection, [1] detections,
 * [2] memory vectors read by association in units of D fp16 values (an fp32 r_frag counts 2),
 * [3] object vector updates, [4] cloud points written, [5] depth pixels read by makeScan,
 * [6] scan points inserted, [7] occupancy cells updated, [8] bytes of host inputs moved to the
 * device by pushes of SMG_MEM_HOST frames (copies plus in-place reads of pinned frames).
 * Returns the number of counters. */
int smg_get_work(smg_batch* b, int64_t* out, int n);

/* ---- standalone occupancy grid + correlative scan matching ---- */
/* GridParams (scenemap grid.hpp:18-21) plus the probability clamp of OccGrid::prob
 * (grid.hpp:75: pmin 0.1, pmax 0.9; unseen cells read pmin). */
typedef struct smg_occ_params {
  float res, l_hit, l_miss, l_min, l_max, pmin, pmax;
} smg_occ_params;

/* Scan2 (scenemap scan.hpp:50-58), host memory: sensor origin, match points (+ optional
 * normals), laser hits (ray end excluded from the misses) and free-ray ends (included), all in
 * the base frame.  Only the laser hits take part in scan matching. */
typedef struct smg_scan2 {
  float ox, oy;
  int32_t n_match;
  const float *mx, *my, *mnx, *mny;
  int32_t n_hit;
  const float *hx, *hy;
  int32_t n_free;
  const float *fx, *fy;
} smg_scan2;

/* Real-time correlative search (the reference configures Cartographer's, slam_carto/config/
 * carto_2d.lua:17-21): offsets of -W..W in x and y in steps of linear_step (must equal the
 * grid resolution: offsets are whole cells), rotations -A..A in steps of angular_step (rad),
 * candidate weight exp(-(|t| * translation_weight + |dth| * rotation_weight)^2). */
typedef struct smg_csm_params {
  double linear_window, angular_window, linear_step, angular_step, translation_weight, rotation_weight;
} smg_csm_params;

typedef struct smg_occ smg_occ;

/* n_maps independent grids, each a fixed window of grid_w x grid_h cells (<= 4096 per side)
 * starting at global cell (grid_x0, grid_y0).  Replaces `OccGrid(p)` (grid.hpp:23), which
 * grows on demand: here a point outside the window fails that grid's insert.  max_points
 * bounds match + hit + free points per scan (<= 65536). */
int smg_occ_create(const smg_occ_params* p, int n_maps, int grid_w, int grid_h, int grid_x0, int grid_y0, int max_points,
                   int dev, smg_occ** out);
int smg_occ_destroy(smg_occ* o);
/* OccGrid::insert(scan, pose) (grid.cpp:95-159) for grids 0..n-1; poses = n x (x, y, th).
 * changed_out (n, or NULL): the reference's return value (cells whose log-odds or seen flag
 * changed), -1 if the scan left the window (the grid is then unchanged).  With changed_out
 * NULL the call is asynchronous on `stream`. */
int smg_occ_insert(smg_occ* o, const smg_scan2* scans, const double* poses, int n, int32_t* changed_out, void* stream);
/* Correlative scan match of each scan's hits around pose0 (n x (x, y, th)) against the
 * current grid: best pose (n x 3), candidate index ((rotation * n_x + x offset) * n_y + y
 * offset, lowest index on ties) and weighted score.  Replaces Cartographer's
 * RealTimeCorrelativeScanMatcher2D::Match as configured by the reference. */
int smg_occ_match(smg_occ* o, const smg_scan2* scans, const double* pose0, const smg_csm_params* c, int n, double* pose_out,
                  int32_t* index_out, double* score_out, void* stream);
/* Match, then insert each scan at its matched pose (one scan-matching front-end step). */
int smg_occ_track(smg_occ* o, const smg_scan2* scans, const double* pose0, const smg_csm_params* c, int n, double* pose_out,
                  int32_t* index_out, double* score_out, int32_t* changed_out, void* stream);
/* Cells of grid m (row-major grid_w x grid_h): log-odds x 256, seen, export8 value (-1
 * unknown, 0..100), and the matcher's quantised probability; any pointer may be NULL. */
int smg_occ_get_cells(smg_occ* o, int m, int16_t* L, uint8_t* seen, int8_t* c8, uint16_t* q);

/* ---- text model: label log-likelihoods and names ---- */
/* apLabelLogLik (objprob.cpp:287-310) for n embeddings z (n x dim, device): out (n x n_labels,
 * device) = per-label log sigma(scale * max row cosine + bias), normalised over the labels;
 * labels without a text row get -1e30.  n_labels <= 1024.  Asynchronous on `stream`. */
int smg_label_loglik(const smg_text* t, const float* z, int n, float* out, void* stream);
/* ApParams naming fields (objprob.hpp:84-87). */
typedef struct smg_name_params {
  double whole_w, name_wmax, size_w, name_tau;
} smg_name_params;
/* apName (objprob.cpp:396-455) for n_obj objects (device arrays, n_obj x n_labels for the L
 * vectors; NULL = that vector is empty in the reference's ApState): Sigma w log p from fragment
 * and whole views (lw_* = their weights), external and geometric log-likelihoods, object size
 * (longest side, m).  Outputs: post (n_obj x n_labels), lab3 = {name_lab, top_lab, rolled} and
 * val3 = {name_p, top_p, name_H} per object; name_lab = -2 when the object has no image
 * evidence (the reference then leaves its name unchanged). */
int smg_name(const smg_text* t, const smg_name_params* p, int n_obj, const float* L_frag, const double* lw_frag,
             const float* L_whole, const double* lw_whole, const float* L_ext, const float* L_geo, const double* size,
             float* post, int32_t* lab3, float* val3, void* stream);

/* ---- association stress ---- */
/* The association step of ObjectMap::update (scenemap objmap.cpp:774-810: box gate, best
 * cosine above the threshold, top-1) in its dense stress form: every detection against a bank
 * of memory vectors.  Embeddings are bf16 (raw uint16 bits), L2-normalised, dim a multiple of
 * 64, rows 16-byte aligned; boxes are float (lo x, y, z, hi x, y, z). */
typedef struct smg_assoc smg_assoc;
int smg_assoc_create(int max_det, int max_mem, int dim, int dev, smg_assoc** out);
int smg_assoc_destroy(smg_assoc* a);
/* For each detection d: the memory j with 3D IoU(box_d, box_j) > iou_min and the largest
 * fp64 dot product (bf16 values, summed in index order) >= cos_min, lowest j on ties, else -1
 * (match[d]); score[d] = that dot product; certified[d] = 1 when the decision was read off the
 * tensor-core scores, 0 when it was recomputed exactly (near the threshold or a near tie).
 * scores (optional, n_det x n_mem fp32): the raw tensor-core dot products.  All pointers are
 * device memory; asynchronous on `stream`. */
int smg_assoc_match(smg_assoc* a, const uint16_t* det, const float* det_box, int n_det, const uint16_t* mem, const float* mem_box,
                    int n_mem, float iou_min, double cos_min, int32_t* match, double* score, int32_t* certified,
                    float* scores, void* stream);
/* Device error word of the batch of matches so far (1 = a pipeline wait timed out). */
int smg_assoc_error(smg_assoc* a);
/* Instrumentation: enable = 1 makes the following matches record %globaltimer at 16 points of
 * one CTA (0 start, 1 TMEM ready, 2 first loads issued, 3 first stage landed, 4 last stage
 * landed, 5 all MMAs done, 6 epilogue done, 7 exit, 8-11 epilogue steps); out16 (or NULL)
 * receives the last record. */
int smg_assoc_stamps(smg_assoc* a, int enable, int64_t* out16);

/* Batched plane fit: replaces scenemap::apPlaneFit (objprob.hpp:204, objprob.cpp:130-209), one
 * call per point set there.  Set s is the float (x, y, z) points xyz[3*off[s] .. 3*off[s+1]),
 * fitted with distance tau and RANSAC seed seeds[s] (apSeed values), at most max_iters
 * (1..256) hypotheses.  out[10*s .. 10*s+9] = ok, n[0..2], thick, inl, zmed, zlo, zhi, hspan;
 * an unfitted set gets the reference's ApPlane defaults (ok 0, n = (0,0,1), thick 1, rest 0)
 * and a set with malformed offsets gets ok = -1.  n_points = off[n_sets].  xyz, off, seeds and
 * out are device memory; the call is asynchronous on `stream`.  Scratch of 16 bytes per point
 * is allocated and freed stream-ordered (cudaMallocAsync) inside the call, and a 1 MB
 * iteration table is allocated once per device on first use. */
int smg_plane_fit(const float* xyz, const int32_t* off, int n_sets, int n_points, double tau, const uint64_t* seeds,
                  int max_iters, double* out, void* stream);

/* smg_plane_fit without any device allocation.  No counterpart in the reference: it exists for
 * callers that cannot allocate device memory while they run, such as a robot's real-time frame
 * loop that reserves all of its GPU memory at start-up (cudaMalloc and cudaMallocAsync can
 * block, synchronise or fail against a fixed memory budget in the middle of a frame) or a
 * plugin host whose per-frame step forbids allocation.  Same arguments and results as
 * smg_plane_fit; the caller still provides xyz, off, seeds and out in device memory.
 * Limit: n_points <= 65536 per call (SMG_ERR_CAPACITY with a message otherwise).  The scratch
 * (1 MiB) and the iteration table (1 MiB) are static device arrays of the library, held on
 * every GPU that loads it until the process exits.  The first call on each device does a
 * one-time set-up on that device (address look-up and a synchronous table copy), so make that
 * first call before any stream capture; after a cudaDeviceReset the next call repeats it.  All calls share the one scratch array: calls that
 * can overlap on the GPU (other streams, other host threads) race and must be serialised by
 * the caller.  Nothing in the scratch needs to start at zero, so no call clears it. */
int smg_plane_fit_noalloc(const float* xyz, const int32_t* off, int n_sets, int n_points, double tau,
                          const uint64_t* seeds, int max_iters, double* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SMG_H */
