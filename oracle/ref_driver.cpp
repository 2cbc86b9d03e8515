// Oracle driver (TEST INFRASTRUCTURE ONLY — never part of the product path).
//
// Drives the reference scenemap C++ code, compiled in place from the reference sources by
// oracle/Makefile into oracle/_ref/libscenemap_ref.so, through its C++ API:
//   Mapper2D::keyframe (scenemap src/mapper2d.cpp:27-87)  -> makeScan + OccGrid::insert
//   ObjectMap::update   (scenemap src/objmap.cpp:516)    -> the objprob per-frame update
//   ObjectMap::addPoints(scenemap src/objmap.cpp:508)    -> ObjCloud::add (cloud.cpp:86)
//   ObjectMap::buildReencode (scenemap src/objmap.cpp:1371) -> whole-object re-encode requests
// in the order the reference's keyframe glue runs them (scenemap src/capi.cpp:811-1010),
// minus robot FK.  With an RGBA image the glue's best-view selection and point colouring
// (capi.cpp:903-998: restated here around the reference's own cropGeometry, cropMask,
// cropRgbHost, cropDepthMm and gatherRgbHost from bestview.cpp) run as well.
// The label image is turned into the sm_detections bit masks the reference consumes
// (scenemap include/scenemap.h:20-34), with the mask grid equal to the image grid.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <memory>
#include <unordered_set>
#include <string>
#include <vector>

#include "scenemap/bestview.hpp"
#include "scenemap/grid.hpp"
#include "scenemap/mapper2d.hpp"
#include "scenemap/objmap.hpp"
#include "scenemap/objprob.hpp"
#include "scenemap/scan.hpp"
#include "scenemap/cloud.hpp"
#include "scenemap/walls.hpp"

using namespace scenemap;

extern "C" {

typedef struct {
  double stamp;
  int w, h;
  const float* depth;
  const uint16_t* label;
  float fx, fy, cx, cy;
  double T_mc[12];
  float T_bc[12];
  double base[3];         // map pose of the base (x, y, th): the grid insert pose
  double eef[2][3];       // hand points, map frame (objprob hand filters)
  float eef_base[2][3];   // hand points, base frame (scan body mask)
  int n_det;
  const uint16_t* det_label;
  const float* box;
  const int32_t* cls;
  const float* score;
  const float* emb;
  int emb_dim;
  int grid_only;          // 1: keyframe only (no detections)
  float grip[2];          // gripper values (ObjFrame::grip; 1 = open)
  // detector bit masks on their own grid (sm_detections), used instead of the label image
  const uint32_t* mask_bits;
  int mask_w, mask_h;
  float mask_sx, mask_sy, mask_ox, mask_oy;
  int img_w, img_h;       // detector image (0 = the depth image's size)
  const uint16_t* depth_mm;   // ObjFrame::depth_mm / DepthView::mm, when depth is null
  const uint8_t* rgba;        // sm_image::rgba (w x h x 4), or null
  const double* wall_segs;    // ObjFrame::wall_segs (n_wall_segs x 4), or null
  int n_wall_segs;
} rf_frame;

typedef struct {
  uint32_t id;
  int32_t cls;
  double pos[3], ext[3], first_pos[3], lo[3], hi[3];
  uint32_t n_obs;
  double first_seen, last_seen;
  int32_t state, confirmed, moved, misses;
  uint32_t n_vis_miss;
  float score;
  double max_det_z, last_kf, gone_t;
  int32_t appeared, mv_cnt;
  double trk_pos[3], trk_t, trk_step[2], moving_t, move_from_t;
  double first_miss, miss_cam[3], last_miss_cam[3], last_miss_fwd[3];
  // cloud
  int32_t cloud_n;
  uint32_t cloud_version;
  double cloud_org[3];
  // objprob state
  uint32_t ap_ver;
  double k_frag, k_whole;
  int32_t n_views, n_ap_obs, n_wall_obs, n_struct_look, need_whole, n_whole;
  double P[3];
  int32_t n_cams, geo;
  int32_t drop, hide;
  int32_t held_by;
  uint32_t parent;
  double parent_rel[3];
  int32_t wall_like;
  float fw;
} rf_obj;

typedef struct {
  long n_through, n_obs, n_wall, n_wall_name, n_ceil, n_floor, n_assoc, n_new, n_merge, n_obj_struct, n_reenc_req, n_reenc_done,
      n_blocked, n_wall_tall, n_so_big, n_bridge;
} rf_stats;

struct RefMap {
  ObjectMap om;
  std::unique_ptr<Mapper2D> mapper;
  KeyframeStats kf;
  std::vector<uint32_t> bits;
  std::vector<ObsPoints> pts;   // copy of lastPoints() as handed to addPoints
  std::vector<ReencReq> reenc;  // re-encode requests of the last keyframe
  int reenc_words = 0;
  bool reenc_on = true;   // build the re-encode requests (the reference's push always does)
  // best views (sm_ctx::views, view_ver, ev_seen: capi.cpp:113-116)
  struct Slot {
    std::shared_ptr<const BestView> v;
    double q = 0;
  };
  std::map<uint32_t, Slot> views;
  uint32_t view_ver = 0;
  size_t ev_seen = 0;
  // wall extraction as sm_push_image runs it before the object update (refreshWalls and the
  // window bridges, capi.cpp:646-698, 866-890: sm_ctx::wallsp, walls_rects, walls_grid_ver,
  // wall_th, wall_th_t, walls_full_t), on the occupancy grid laid over a fixed window of cells
  // [wx0, wx0 + ww) x [wy0, wy0 + wh) (the device library's grid window)
  bool walls_on = false;
  int wx0 = 0, wy0 = 0, ww = 0, wh = 0;
  std::vector<int8_t> wgrid;
  std::shared_ptr<const std::vector<WallSeg>> wallsp;
  std::vector<WallRect> walls_rects;
  uint64_t walls_grid_ver = ~0ull;
  double wall_th = 0, wall_th_t = -1e300, walls_full_t = -1e300;
  std::vector<double> wsegs;
  explicit RefMap(const ObjParams& p) : om(p) {}
};

// export8 of the reference grid laid over the window (cells outside the grid: -1 unknown);
// false when a seen cell of the grid lies outside the window
static bool window_grid(RefMap* m) {
  const OccGrid& G = m->mapper->grid();
  m->wgrid.assign(size_t(m->ww) * m->wh, int8_t(-1));
  if (G.width() <= 0 || G.height() <= 0) return true;
  const std::vector<int8_t> c8 = G.export8();
  bool ok = true;
  for (int y = 0; y < G.height(); ++y)
    for (int x = 0; x < G.width(); ++x) {
      const int8_t v = c8[size_t(y) * G.width() + x];
      const int gx = G.x0() + x - m->wx0, gy = G.y0() + y - m->wy0;
      if (gx < 0 || gy < 0 || gx >= m->ww || gy >= m->wh) { ok = ok && v < 0; continue; }
      m->wgrid[size_t(gy) * m->ww + gx] = v;
    }
  return ok;
}

static WallGrid window_view(const RefMap* m) {
  const double res = double(m->mapper->grid().res());
  return WallGrid{m->wgrid.data(), m->ww, m->wh, res, m->wx0 * res, m->wy0 * res};
}

// refreshWalls (capi.cpp:646-698) and the bridged segment list of the keyframe (:866-890)
static int refresh_walls(RefMap* m, double now) {
  if (!window_grid(m)) return -2;
  const OccGrid& gr = m->mapper->grid();
  const bool grid_changed = m->walls_grid_ver != gr.cellsVersion();
  std::vector<WallRect> rects;
  for (const MapObject& o : m->om.objects()) {
    if (!m->om.exportable(o) || o.held_by >= 0 || o.state == SM_GONE) continue;
    if (o.lo[2] > 0.4) continue;
    if (o.ap && o.ap->wall_like) continue;
    if (m->om.kindOf(o.cls) == kKindStructObj) continue;
    const double dx = o.hi[0] - o.lo[0], dy = o.hi[1] - o.lo[1];
    if (dx > 5.0 || dy > 5.0) continue;
    rects.push_back({o.lo[0] - 0.1, o.lo[1] - 0.1, o.hi[0] + 0.1, o.hi[1] + 0.1});
  }
  const bool rects_changed = !(rects == m->walls_rects);
  const WallGrid wg = window_view(m);
  bool th_changed = false;
  if ((grid_changed || rects_changed) && now - m->wall_th_t >= 2.0) {
    const double th = wallAngle(wg, &rects);
    m->wall_th_t = now;
    if (std::abs(th - m->wall_th) > M_PI / 180.0) {
      const bool was_axis = std::abs(m->wall_th) <= kAlignTol, is_axis = std::abs(th) <= kAlignTol;
      if (was_axis != is_axis) m->wallsp.reset();
      m->wall_th = th;
      th_changed = true;
    }
  }
  bool redo;
  if (std::abs(m->wall_th) > kAlignTol)
    redo = !(m->wallsp && !th_changed && !rects_changed && (!grid_changed || now - m->walls_full_t < 0.5));
  else
    redo = !(m->wallsp && !grid_changed && !rects_changed);
  if (redo) {
    // the incremental extractor of the axis-aligned case returns what wallSegments does
    m->wallsp = std::make_shared<const std::vector<WallSeg>>(
        std::abs(m->wall_th) > kAlignTol ? wallSegmentsAtAngle(wg, m->wall_th, kMinLen, kMaxThick, 0.6, &rects)
                                         : wallSegments(wg, kMinLen, kMaxThick, 0.6, &rects));
    m->walls_rects = std::move(rects);
    m->walls_grid_ver = gr.cellsVersion();
    if (std::abs(m->wall_th) > kAlignTol) m->walls_full_t = now;
  }
  m->wsegs.clear();
  if (m->wallsp) {
    const auto& W = *m->wallsp;
    for (const WallSeg& w : W) m->wsegs.insert(m->wsegs.end(), {w.ax, w.ay, w.bx, w.by});
    const double bmax = m->om.params().ap.bridge_max;
    for (size_t i = 0; i < W.size(); ++i)
      for (size_t j = i + 1; j < W.size(); ++j) {
        const double ux = W[i].bx - W[i].ax, uy = W[i].by - W[i].ay, li = std::hypot(ux, uy);
        const double vx = W[j].bx - W[j].ax, vy = W[j].by - W[j].ay, lj = std::hypot(vx, vy);
        if (li < 1e-6 || lj < 1e-6 || std::fabs(ux * vy - uy * vx) / (li * lj) > 0.03) continue;
        const double nx = -uy / li, ny = ux / li;
        if (std::fabs((W[j].ax - W[i].ax) * nx + (W[j].ay - W[i].ay) * ny) > 0.1) continue;
        auto at = [&](double x, double y) { return ((x - W[i].ax) * ux + (y - W[i].ay) * uy) / li; };
        double a0 = 0, a1 = li, b0 = at(W[j].ax, W[j].ay), b1 = at(W[j].bx, W[j].by);
        if (b0 > b1) std::swap(b0, b1);
        const double lo = a1 <= b0 ? a1 : b1, hi = a1 <= b0 ? b0 : a0;
        if (hi - lo <= 0 || hi - lo > bmax) continue;
        m->wsegs.insert(m->wsegs.end(), {W[i].ax + ux / li * lo, W[i].ay + uy / li * lo, W[i].ax + ux / li * hi, W[i].ay + uy / li * hi});
      }
  }
  return 0;
}

void* ref_create(const char* obj_kv, double voxel, int cloud_cap, int grid_on, const float* grid /* res, l_hit, l_miss, l_min, l_max */,
                 int attach_on) {
  ObjParams p;
  if (obj_kv && *obj_kv) ObjectMap::applyParams(&p, obj_kv, false);
  if (voxel > 0) p.voxel = voxel;
  if (cloud_cap > 0) p.cloud_cap = cloud_cap;
  RefMap* m = new RefMap(p);
  if (grid_on) {
    MapperParams mp;
    if (grid) {
      mp.grid.res = grid[0];
      mp.grid.l_hit = grid[1];
      mp.grid.l_miss = grid[2];
      mp.grid.l_min = grid[3];
      mp.grid.l_max = grid[4];
    }
    mp.attach.enabled = attach_on != 0;
    m->mapper.reset(new Mapper2D(mp));
  }
  return m;
}

void ref_destroy(void* h) { delete static_cast<RefMap*>(h); }

// sm_snapshot's object list (capi.cpp:1051-1067; big = ObjParams::big): the exportable objects
// in object order.  Record layout of smg_snap_object.
typedef struct {
  uint32_t id;
  int32_t name_lab;
  float score;
  double pos[3], extent[3], first_pos[3];
  uint32_t n_obs;
  double last_seen;
  int32_t state, structural, movable, n_points;
  double cloud_stamp;
} rf_snap;

int ref_snapshot(void* h, rf_snap* out, int cap) {
  RefMap* m = static_cast<RefMap*>(h);
  const double big = m->om.params().big;
  int n = 0;
  for (const MapObject& o : m->om.objects()) {
    if (!m->om.exportable(o)) continue;
    if (out && n < cap) {
      rf_snap& e = out[n];
      memset(&e, 0, sizeof(e));
      e.id = o.id;
      e.name_lab = o.cls;   // the label index (the runtime names it from its label table)
      e.score = o.score;
      for (int k = 0; k < 3; ++k) { e.pos[k] = o.pos[k]; e.extent[k] = o.ext[k]; e.first_pos[k] = o.first_pos[k]; }
      e.n_obs = o.n_obs;
      e.last_seen = o.last_seen;
      e.state = o.held_by >= 0 ? SM_HELD : o.state;
      const int kind = m->om.kindOf(o.cls);
      e.structural = kind == kKindStatic || kind == kKindStructObj || std::max({o.ext[0], o.ext[1], o.ext[2]}) > big;
      e.movable = kind != kKindStatic && kind != kKindStructObj;
      e.n_points = int(o.cloud.size());
      e.cloud_stamp = o.cloud.stamp;
    }
    ++n;
  }
  return n;
}

// dsg_save.cpp:70-89 plyBytes of the n-th exportable object: the whole file (header and 15-byte
// vertex records); returns its size
long ref_snapshot_ply(void* h, int n, uint8_t* out, long cap) {
  RefMap* m = static_cast<RefMap*>(h);
  int k = -1;
  for (const MapObject& o : m->om.objects()) {
    if (!m->om.exportable(o) || ++k != n) continue;
    const ObjCloud& c = o.cloud;
    const size_t np = c.size();
    std::string hdr = "ply\nformat binary_little_endian 1.0\nelement vertex " + std::to_string(np) +
                      "\nproperty float x\nproperty float y\nproperty float z\nproperty uchar red\nproperty uchar green\n"
                      "property uchar blue\nend_header\n";
    const long total = long(hdr.size() + np * 15);
    if (!out || cap < total) return total;
    memcpy(out, hdr.data(), hdr.size());
    uint8_t* p = out + hdr.size();
    for (size_t i = 0; i < np; ++i, p += 15) {
      const CloudPt& q = c.data->pts[i];
      const float xyz[3] = {float(c.org[0] + q.x), float(c.org[1] + q.y), float(c.org[2] + q.z)};
      memcpy(p, xyz, 12);
      p[12] = q.r;
      p[13] = q.g;
      p[14] = q.b;
    }
    return total;
  }
  return -1;
}

// Wall extraction before every object update (sm_push_image's refreshWalls), on the grid window
// x0, y0 (cells), w x h.
int ref_set_walls(void* h, int on, int x0, int y0, int w, int hh) {
  RefMap* m = static_cast<RefMap*>(h);
  if (!m || !m->mapper || w <= 0 || hh <= 0) return -1;
  m->walls_on = on != 0;
  m->wx0 = x0; m->wy0 = y0; m->ww = w; m->wh = hh;
  return 0;
}

// sm_snap_wall_segments (capi.cpp:1247-1257): the extracted segments (no bridges), count or -1
int ref_wall_segments(void* h, double* out, int cap) {
  RefMap* m = static_cast<RefMap*>(h);
  if (!m || !m->wallsp) return -1;
  const auto& W = *m->wallsp;
  for (int i = 0; out && i < cap && i < int(W.size()); ++i) {
    out[4 * i] = W[i].ax; out[4 * i + 1] = W[i].ay; out[4 * i + 2] = W[i].bx; out[4 * i + 3] = W[i].by;
  }
  return int(W.size());
}

// sm_snap_wall_state (capi.cpp:1239-1245) on the window grid: kStateLen floats
int ref_wall_state(void* h, const double pose[3], float* out) {
  RefMap* m = static_cast<RefMap*>(h);
  if (!m || !m->wallsp || !window_grid(m)) return -1;
  wallStateVector(window_view(m), *m->wallsp, pose, out);
  return 0;
}

// the wall-extraction functions on a caller's grid (walls.hpp): wallSegments / wallAngle /
// wallSegmentsAtAngle, for tests of the extraction alone
int ref_wall_segments_grid(const int8_t* cells, int w, int hh, double res, double ox, double oy, const double* rects, int n_rects,
                           int mode, double th, double* angle_out, double* out, int cap) {
  const WallGrid g{cells, w, hh, res, ox, oy};
  std::vector<WallRect> rv;
  for (int i = 0; i < n_rects; ++i) rv.push_back({rects[4 * i], rects[4 * i + 1], rects[4 * i + 2], rects[4 * i + 3]});
  std::vector<WallSeg> W;
  if (mode == 0) W = wallSegments(g, kMinLen, kMaxThick, 0.6, &rv);
  else if (mode == 1) { const double a = wallAngle(g, &rv); if (angle_out) *angle_out = a; return 0; }
  else W = wallSegmentsAtAngle(g, th, kMinLen, kMaxThick, 0.6, &rv);
  for (int i = 0; out && i < cap && i < int(W.size()); ++i) {
    out[4 * i] = W[i].ax; out[4 * i + 1] = W[i].ay; out[4 * i + 2] = W[i].bx; out[4 * i + 3] = W[i].by;
  }
  return int(W.size());
}

// Skip buildReencode (to time the keyframe without the re-encode stage, as the device can).
void ref_set_reencode(void* h, int on) { static_cast<RefMap*>(h)->reenc_on = on != 0; }

int ref_frame(void* h, const rf_frame* f) {
  RefMap* m = static_cast<RefMap*>(h);
  if (!m || !f || f->w <= 0 || f->h <= 0 || (!f->depth && !f->depth_mm)) return -1;
  if (m->mapper) {   // Mapper2D::keyframe as capi.cpp:809-820 sets it up (no FK capsules)
    DepthView dv;
    dv.w = f->w;
    dv.h = f->h;
    dv.m = f->depth;
    dv.mm = f->depth ? nullptr : f->depth_mm;
    dv.step = std::max(1, int(std::lround(f->w / 160.0)));
    dv.fx = f->fx; dv.fy = f->fy; dv.cx = f->cx; dv.cy = f->cy;
    memcpy(dv.T_bc, f->T_bc, sizeof(dv.T_bc));
    BodyState b;
    for (int s = 0; s < 2; ++s) for (int k = 0; k < 3; ++k) b.eef[s][k] = f->eef_base[s][k];
    Pose2 known{f->base[0], f->base[1], f->base[2]};
    m->kf = m->mapper->keyframe(dv, b, known, nullptr);
  }
  m->reenc.clear();
  if (f->grid_only) return 0;
  if (m->walls_on) {
    if (f->wall_segs || !m->mapper) return -1;
    if (int r = refresh_walls(m, f->stamp)) return r;
  }
  // detections: the caller's bit masks, or the label image turned into bit masks on the image
  // grid (sm_detections, scenemap include/scenemap.h:20-34)
  const int n = f->n_det;
  const int img_w = f->img_w > 0 ? f->img_w : f->w, img_h = f->img_h > 0 ? f->img_h : f->h;
  sm_detections d;
  memset(&d, 0, sizeof(d));
  d.stamp = f->stamp;
  d.img_w = img_w;
  d.img_h = img_h;
  d.n = n;
  d.cls = f->cls;
  d.score = f->score;
  d.box = f->box;
  if (f->mask_bits) {
    d.mask_w = f->mask_w;
    d.mask_h = f->mask_h;
    d.mask_sx = f->mask_sx;
    d.mask_sy = f->mask_sy;
    d.mask_ox = f->mask_ox;
    d.mask_oy = f->mask_oy;
    d.mask_bits = f->mask_bits;
  } else {
    const size_t words = (size_t(f->w) * f->h + 31) / 32;
    m->bits.assign(words * size_t(std::max(0, n)), 0u);
    std::vector<size_t> slot(65536, SIZE_MAX);
    for (int k = 0; k < n; ++k) slot[f->det_label[k]] = size_t(k);
    if (f->label)
      for (size_t c = 0; c < size_t(f->w) * f->h; ++c) {
        const size_t k = slot[f->label[c]];
        if (k != SIZE_MAX) m->bits[k * words + (c >> 5)] |= 1u << (c & 31);
      }
    d.mask_w = f->w;
    d.mask_h = f->h;
    d.mask_sx = d.mask_sy = 1.f;
    d.mask_ox = d.mask_oy = 0.f;
    d.mask_bits = m->bits.data();
  }
  ObjFrame F;
  F.stamp = f->stamp;
  F.w = f->w;
  F.h = f->h;
  F.depth_m = f->depth;
  F.depth_mm = f->depth ? nullptr : f->depth_mm;
  F.fx = f->fx; F.fy = f->fy; F.cx = f->cx; F.cy = f->cy;
  memcpy(F.T_mc, f->T_mc, sizeof(F.T_mc));
  F.dets = n > 0 ? &d : nullptr;
  for (int s = 0; s < 2; ++s) for (int k = 0; k < 3; ++k) F.eef[s][k] = f->eef[s][k];
  F.grip[0] = f->grip[0];
  F.grip[1] = f->grip[1];
  F.base_yaw = f->base[2];
  F.base_xy[0] = f->base[0];
  F.base_xy[1] = f->base[1];
  F.emb = f->emb;
  F.emb_dim = f->emb_dim;
  F.wall_segs = f->wall_segs;
  F.n_wall_segs = f->n_wall_segs;
  if (m->walls_on) {   // an empty list is a null pointer there (a fresh vector)
    F.wall_segs = m->wsegs.empty() ? nullptr : m->wsegs.data();
    F.n_wall_segs = int(m->wsegs.size() / 4);
  }
  m->om.update(F);
  // best views (capi.cpp:903-943): moved / put-down events reset the view quality, views of
  // objects that are gone are dropped, detections attached to an object become candidates
  const auto& ev = m->om.events();
  for (; m->ev_seen < ev.size(); ++m->ev_seen)
    if (ev[m->ev_seen].kind == 2 || ev[m->ev_seen].kind == 5) {
      auto it = m->views.find(ev[m->ev_seen].id);
      if (it != m->views.end()) it->second.q = 0;
    }
  if (!m->views.empty()) {
    std::unordered_set<uint32_t> live;
    for (const MapObject& o : m->om.objects()) live.insert(o.id);
    for (auto it = m->views.begin(); it != m->views.end();) it = live.count(it->first) ? std::next(it) : m->views.erase(it);
  }
  const bool host_rgb = f->rgba && d.img_w == f->w && d.img_h == f->h;
  struct Cand {
    uint32_t id;
    double q;
    std::shared_ptr<BestView> v;
  };
  std::vector<Cand> cand;
  const std::vector<DetAssoc>& as = m->om.lastAssoc();
  for (size_t k = 0; k < as.size() && host_rgb; ++k) {
    if (!as[k].obj_id) continue;
    const float sc = d.score ? d.score[k] : 1.f;
    const double q = double(as[k].area_px) * sc;
    auto it = m->views.find(as[k].obj_id);
    if (it != m->views.end() && q < it->second.q) continue;
    auto v = std::make_shared<BestView>();
    const float* b = d.box + 4 * k;
    if (!cropGeometry(b, d.img_w, d.img_h, 0.10f, 256, v->box, &v->w, &v->h)) continue;   // kCropMargin, kCropMaxSide
    v->id = as[k].obj_id;
    v->q = q;
    v->stamp = f->stamp;
    for (int i = 0; i < 4; ++i) v->det_box[i] = int32_t(std::lround(b[i]));
    v->mask_area = as[k].area_px;
    v->depth_m = as[k].depth_med;
    v->score = sc;
    memcpy(v->cam_T, F.T_mc, sizeof(v->cam_T));
    v->rgb.resize(size_t(v->w) * v->h * 3);
    v->depth.resize(size_t(v->w) * v->h);
    cropMask(&d, int(k), v->box, v->w, v->h, &v->mask);
    cand.push_back(Cand{v->id, q, std::move(v)});
  }
  // cloud points, coloured from the image when there is one (capi.cpp:944-956, :986-992)
  m->pts = m->om.lastPoints();
  size_t npt = 0;
  for (const ObsPoints& q : m->pts) npt += q.px.size() / 2;
  std::vector<int32_t> xy;
  std::vector<uint8_t> rgb;
  if (npt && host_rgb) {
    xy.reserve(2 * npt);
    for (const ObsPoints& q : m->pts) xy.insert(xy.end(), q.px.begin(), q.px.end());
    rgb.assign(3 * npt, 128);
    gatherRgbHost(f->rgba, int64_t(f->w) * 4, 4, f->w, f->h, xy.data(), int(npt), rgb.data());
  }
  // crops (capi.cpp:958-972); depth from the frame's metres (millimetre frames: mm * 1e-3f)
  std::vector<float> dm;
  const float* depth_m = f->depth;
  if (!depth_m && !cand.empty()) {
    dm.resize(size_t(f->w) * f->h);
    for (size_t i = 0; i < dm.size(); ++i) dm[i] = float(f->depth_mm[i]) * 1e-3f;
    depth_m = dm.data();
  }
  for (Cand& c : cand) {
    const sm_crop_req r{c.v->box[0], c.v->box[1], c.v->box[2], c.v->box[3], c.v->w, c.v->h, c.v->rgb.data()};
    cropRgbHost(f->rgba, int64_t(f->w) * 4, 4, r);
    cropDepthMm(depth_m, f->w, f->h, d.img_w, d.img_h, c.v->box, c.v->w, c.v->h, c.v->depth.data());
  }
  size_t off = 0;
  for (const ObsPoints& q : m->pts) {
    const int np = int(q.px.size() / 2);
    m->om.addPoints(q.obj_id, q.xyz.data(), host_rgb ? rgb.data() + 3 * off : nullptr, np, f->stamp);
    off += size_t(np);
  }
  // installs (capi.cpp:994-998)
  for (Cand& c : cand) {
    RefMap::Slot& sl = m->views[c.id];
    if (sl.v && c.q < sl.q) continue;
    c.v->version = ++m->view_ver;
    sl.v = std::move(c.v);
    sl.q = c.q;
  }
  // whole-object re-encode requests on frames with detection embeddings (capi.cpp:1002-1005),
  // the mask grid being the image grid
  if (n > 0 && f->emb && m->reenc_on)
    m->om.buildReencode(F, d.img_w, d.img_h, d.mask_w, d.mask_h, d.mask_sx, d.mask_sy, d.mask_ox, d.mask_oy, &m->reenc);
  m->reenc_words = int((size_t(d.mask_w) * d.mask_h + 31) / 32);
  return 0;
}

// Re-encode requests of the last keyframe: id, box (4), kappa, cam (6) and the mask bits
// (words_per_request words each, consecutive).  Returns the count; copies up to cap.
int ref_reenc(void* h, uint32_t* id, float* box, float* kappa, double* cam, uint32_t* bits, int cap) {
  RefMap* m = static_cast<RefMap*>(h);
  const int n = int(m->reenc.size());
  for (int r = 0; r < n && r < cap; ++r) {
    const ReencReq& q = m->reenc[r];
    if (id) id[r] = q.id;
    if (box) for (int k = 0; k < 4; ++k) box[4 * r + k] = q.box[k];
    if (kappa) kappa[r] = q.kappa;
    if (cam) for (int k = 0; k < 6; ++k) cam[6 * r + k] = q.cam[k];
    if (bits)
      for (int k = 0; k < m->reenc_words; ++k) bits[size_t(r) * m->reenc_words + k] = k < int(q.bits.size()) ? q.bits[k] : 0u;
  }
  return n;
}
int ref_reenc_words(void* h) { return static_cast<RefMap*>(h)->reenc_words; }

// The caller's answer to the requests (sm_set_object_embeddings, scenemap capi.cpp:1825-1835):
// whole-object embedding i of object ids[i] is added with the kappa and camera of its request,
// at the request frame's stamp; ids without a request are skipped.  Returns the number added.
int ref_add_whole_views(void* h, const uint32_t* ids, const float* emb, int n, int dim, double stamp) {
  RefMap* m = static_cast<RefMap*>(h);
  int added = 0;
  for (int i = 0; i < n; ++i) {
    const ReencReq* r = nullptr;
    for (const ReencReq& q : m->reenc) if (q.id == ids[i]) { r = &q; break; }
    if (!r) continue;
    m->om.addWholeView(ids[i], emb + size_t(i) * dim, dim, r->kappa, stamp, r->cam);
    ++added;
  }
  return added;
}

// r_whole of object i (zeros when it has none) and k_whole; returns n_whole (-1: no object)
int ref_object_whole(void* h, int i, float* r_whole, int D, double* k_whole) {
  const auto& objs = static_cast<RefMap*>(h)->om.objects();
  if (i < 0 || size_t(i) >= objs.size() || !objs[size_t(i)].ap) return -1;
  const ApState& s = *objs[size_t(i)].ap;
  for (int k = 0; k < D; ++k) r_whole[k] = size_t(k) < s.r_whole.size() ? s.r_whole[size_t(k)] : 0.f;
  *k_whole = s.k_whole;
  return s.r_whole.empty() ? 0 : s.n_whole;
}

int ref_n_objects(void* h) { return int(static_cast<RefMap*>(h)->om.objects().size()); }

int ref_objects(void* h, rf_obj* out, int cap) {
  const auto& objs = static_cast<RefMap*>(h)->om.objects();
  const int n = std::min<int>(cap, int(objs.size()));
  for (int i = 0; i < n; ++i) {
    const MapObject& o = objs[size_t(i)];
    rf_obj& r = out[i];
    memset(&r, 0, sizeof(r));
    r.id = o.id;
    r.cls = o.cls;
    for (int k = 0; k < 3; ++k) {
      r.pos[k] = o.pos[k]; r.ext[k] = o.ext[k]; r.first_pos[k] = o.first_pos[k]; r.lo[k] = o.lo[k]; r.hi[k] = o.hi[k];
      r.trk_pos[k] = o.trk_pos[k]; r.miss_cam[k] = o.miss_cam[k]; r.last_miss_cam[k] = o.last_miss_cam[k];
      r.last_miss_fwd[k] = o.last_miss_fwd[k]; r.cloud_org[k] = o.cloud.org[k];
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
    r.gone_t = o.gone_t;
    r.appeared = o.appeared;
    r.mv_cnt = o.mv_cnt;
    r.trk_t = o.trk_t;
    r.trk_step[0] = o.trk_step[0];
    r.trk_step[1] = o.trk_step[1];
    r.moving_t = o.moving_t;
    r.move_from_t = o.move_from_t;
    r.first_miss = o.first_miss;
    r.cloud_n = int(o.cloud.size());
    r.cloud_version = o.cloud.version;
    r.held_by = o.held_by;
    r.parent = o.parent;
    for (int k = 0; k < 3; ++k) r.parent_rel[k] = o.parent_rel[k];
    if (o.ap) {
      const ApState& s = *o.ap;
      r.ap_ver = s.ver;
      r.k_frag = s.k_frag;
      r.k_whole = s.k_whole;
      r.n_views = int(s.views.size());
      r.n_ap_obs = s.n_ap_obs;
      r.n_wall_obs = s.n_wall_obs;
      r.n_struct_look = s.n_struct_look;
      r.need_whole = s.need_whole;
      r.n_whole = s.n_whole;
      for (int k = 0; k < 3; ++k) r.P[k] = s.P[k];
      r.n_cams = int(s.cams.size());
      r.geo = s.geo;
      r.drop = s.drop;
      r.hide = s.hide;
      r.wall_like = s.wall_like;
      r.fw = s.fw;
    }
  }
  return n;
}

// objprob vectors of object i: r_frag (D floats), views (up to 5: D fp16 each, kappa, stamp)
int ref_object_vectors(void* h, int i, float* r_frag, int D, uint16_t* views, float* vkappa, double* vstamp, int vcap) {
  const auto& objs = static_cast<RefMap*>(h)->om.objects();
  if (i < 0 || size_t(i) >= objs.size() || !objs[size_t(i)].ap) return -1;
  const ApState& s = *objs[size_t(i)].ap;
  if (r_frag) {
    for (int k = 0; k < D; ++k) r_frag[k] = size_t(k) < s.r_frag.size() ? s.r_frag[size_t(k)] : 0.f;
  }
  const int nv = std::min<int>(vcap, int(s.views.size()));
  for (int v = 0; v < nv; ++v) {
    const ApView& w = s.views[size_t(v)];
    if (views) for (int k = 0; k < D; ++k) views[size_t(v) * D + k] = size_t(k) < w.z.size() ? w.z[size_t(k)] : 0;
    if (vkappa) vkappa[v] = w.kappa;
    if (vstamp) vstamp[v] = w.stamp;
  }
  return nv;
}

// cloud of object i in map coordinates (float(org + p), as the reference reads it back) and seq
int ref_object_cloud(void* h, int i, float* xyz, uint32_t* seq, int cap) {
  const auto& objs = static_cast<RefMap*>(h)->om.objects();
  if (i < 0 || size_t(i) >= objs.size()) return -1;
  const MapObject& o = objs[size_t(i)];
  if (!o.cloud.data) return 0;
  const auto& pts = o.cloud.data->pts;
  const int n = std::min<int>(cap, int(pts.size()));
  for (int k = 0; k < n; ++k) {
    if (xyz) {
      xyz[3 * k] = pts[size_t(k)].x;
      xyz[3 * k + 1] = pts[size_t(k)].y;
      xyz[3 * k + 2] = pts[size_t(k)].z;
    }
    if (seq) seq[k] = pts[size_t(k)].seq;
  }
  return int(pts.size());
}

// Text model and class kinds (ObjectMap::setTextModel, setClassKinds; what sm_set_labels,
// sm_set_text_model and sm_set_label_stats install, capi.cpp:1769-1806).  Per-label arrays may be
// null; so_shape and flat_ok are the tables the glue derives from label names.
int ref_set_text_model(void* h, const float* text, const int32_t* row_label, int rows, int dim, float scale, float bias, int n_labels,
                       const float* log_prior, const float* ls_mu, const float* ls_sd, const int32_t* parent, int object_label,
                       const uint8_t* kinds, const uint8_t* so_shape, const uint8_t* flat_ok) {
  RefMap* m = static_cast<RefMap*>(h);
  if (!m || n_labels <= 0 || rows < 0) return -1;
  ApText t;
  t.dim = rows > 0 ? dim : 0;
  if (rows > 0) {
    t.text.assign(text, text + size_t(rows) * dim);
    t.row_label.assign(row_label, row_label + rows);
  }
  t.scale = scale;
  t.bias = bias;
  t.n_labels = n_labels;
  if (log_prior) t.log_prior.assign(log_prior, log_prior + n_labels);
  if (ls_mu && ls_sd) { t.ls_mu.assign(ls_mu, ls_mu + n_labels); t.ls_sd.assign(ls_sd, ls_sd + n_labels); }
  if (parent) t.parent.assign(parent, parent + n_labels);
  t.object_label = object_label;
  if (so_shape) t.so_shape.assign(so_shape, so_shape + n_labels);
  if (flat_ok) t.flat_ok.assign(flat_ok, flat_ok + n_labels);
  m->om.setTextModel(std::move(t));
  if (kinds) m->om.setClassKinds(std::vector<uint8_t>(kinds, kinds + n_labels));
  return 0;
}

// Name state of object i: post (n_labels floats; zeros when empty), lab3 = name_lab, top_lab,
// rolled; val3 = name_p, top_p, name_H.  Returns the post size.
int ref_object_name(void* h, int i, float* post, int n_labels, int32_t* lab3, float* val3) {
  const auto& objs = static_cast<RefMap*>(h)->om.objects();
  if (i < 0 || size_t(i) >= objs.size() || !objs[size_t(i)].ap) return -1;
  const ApState& s = *objs[size_t(i)].ap;
  for (int c = 0; c < n_labels && post; ++c) post[c] = size_t(c) < s.post.size() ? s.post[size_t(c)] : 0.f;
  if (lab3) { lab3[0] = s.name_lab; lab3[1] = s.top_lab; lab3[2] = s.rolled; }
  if (val3) { val3[0] = s.name_p; val3[1] = s.top_p; val3[2] = s.name_H; }
  return int(s.post.size());
}

// Cloud colours of object i (3 bytes a point, the order of ref_object_cloud).
int ref_object_cloud_rgb(void* h, int i, uint8_t* rgb, int cap) {
  const auto& objs = static_cast<RefMap*>(h)->om.objects();
  if (i < 0 || size_t(i) >= objs.size()) return -1;
  const MapObject& o = objs[size_t(i)];
  if (!o.cloud.data) return 0;
  const auto& pts = o.cloud.data->pts;
  const int n = std::min<int>(cap, int(pts.size()));
  for (int k = 0; k < n && rgb; ++k) {
    rgb[3 * k] = pts[size_t(k)].r;
    rgb[3 * k + 1] = pts[size_t(k)].g;
    rgb[3 * k + 2] = pts[size_t(k)].b;
  }
  return int(pts.size());
}

// The views map, by ascending id: id, version, q, stamp, box (4), det_box (4), mask_area,
// depth_m, score, cam_T (12), w, h per view; images at a fixed stride of 256*256 pixels.
typedef struct {
  uint32_t id, version;
  double q, stamp;
  int32_t box[4], det_box[4];
  float mask_area, depth_m, score;
  double cam_T[12];
  int32_t w, h;
} rf_view;
int ref_views(void* h, rf_view* out, uint8_t* rgb, uint16_t* depth, uint8_t* mask, int cap) {
  RefMap* m = static_cast<RefMap*>(h);
  int n = 0;
  for (const auto& kv : m->views) {
    if (!kv.second.v) continue;
    if (n < cap) {
      const BestView& v = *kv.second.v;
      if (out) {
        rf_view& o = out[n];
        memset(&o, 0, sizeof(o));
        o.id = v.id;
        o.version = v.version;
        o.q = v.q;
        o.stamp = v.stamp;
        for (int c = 0; c < 4; ++c) { o.box[c] = v.box[c]; o.det_box[c] = v.det_box[c]; }
        o.mask_area = v.mask_area;
        o.depth_m = v.depth_m;
        o.score = v.score;
        memcpy(o.cam_T, v.cam_T, sizeof(o.cam_T));
        o.w = v.w;
        o.h = v.h;
      }
      const size_t S = 256 * 256;
      if (rgb && !v.rgb.empty()) memcpy(rgb + size_t(n) * S * 3, v.rgb.data(), v.rgb.size());
      if (depth && !v.depth.empty()) memcpy(depth + size_t(n) * S, v.depth.data(), v.depth.size() * 2);
      if (mask && !v.mask.empty()) memcpy(mask + size_t(n) * S, v.mask.data(), v.mask.size());
    }
    ++n;
  }
  return n;
}

// per detection: obj_id, n_valid, area_px, depth_med (ObjectMap::lastAssoc)
int ref_assoc(void* h, uint32_t* obj_id, int32_t* n_valid, float* area_px, float* depth_med, int cap) {
  const auto& as = static_cast<RefMap*>(h)->om.lastAssoc();
  const int n = std::min<int>(cap, int(as.size()));
  for (int k = 0; k < n; ++k) {
    obj_id[k] = as[size_t(k)].obj_id;
    n_valid[k] = as[size_t(k)].n_valid;
    area_px[k] = as[size_t(k)].area_px;
    depth_med[k] = as[size_t(k)].depth_med;
  }
  return int(as.size());
}

// observation cloud candidates of the last update, in emission order
int ref_n_points(void* h) { return int(static_cast<RefMap*>(h)->pts.size()); }
int ref_points(void* h, int j, uint32_t* obj_id, int32_t* det, float* xyz, int32_t* px, int cap) {
  const auto& P = static_cast<RefMap*>(h)->pts;
  if (j < 0 || size_t(j) >= P.size()) return -1;
  const ObsPoints& q = P[size_t(j)];
  const int n = int(q.px.size() / 2);
  if (obj_id) *obj_id = q.obj_id;
  if (det) *det = q.det;
  for (int k = 0; k < std::min(n, cap); ++k) {
    if (xyz) for (int c = 0; c < 3; ++c) xyz[3 * k + c] = q.xyz[size_t(3 * k + c)];
    if (px) for (int c = 0; c < 2; ++c) px[2 * k + c] = q.px[size_t(2 * k + c)];
  }
  return n;
}

void ref_stats(void* h, rf_stats* s) {
  const ApStats& a = static_cast<RefMap*>(h)->om.apStats();
  s->n_through = a.n_through; s->n_obs = a.n_obs; s->n_wall = a.n_wall; s->n_wall_name = a.n_wall_name; s->n_ceil = a.n_ceil;
  s->n_floor = a.n_floor; s->n_assoc = a.n_assoc; s->n_new = a.n_new; s->n_merge = a.n_merge; s->n_obj_struct = a.n_obj_struct;
  s->n_reenc_req = a.n_reenc_req; s->n_reenc_done = a.n_reenc_done; s->n_blocked = a.n_blocked; s->n_wall_tall = a.n_wall_tall;
  s->n_so_big = a.n_so_big; s->n_bridge = a.n_bridge;
}

int ref_n_events(void* h) { return int(static_cast<RefMap*>(h)->om.events().size()); }
int ref_events(void* h, double* t, uint32_t* id, int32_t* kind, int cap) {
  const auto& ev = static_cast<RefMap*>(h)->om.events();
  const int n = std::min<int>(cap, int(ev.size()));
  for (int k = 0; k < n; ++k) { t[k] = ev[size_t(k)].t; id[k] = ev[size_t(k)].id; kind[k] = ev[size_t(k)].kind; }
  return int(ev.size());
}

// keyframe stats of the last frame: inserted, changed_cells, n_hits
void ref_kf(void* h, int32_t* out3) {
  const KeyframeStats& k = static_cast<RefMap*>(h)->kf;
  out3[0] = k.inserted;
  out3[1] = k.changed_cells;
  out3[2] = k.n_hits;
}

// grid geometry (x0, y0, w, h) and per-cell log-odds (1/256 fixed point), seen flag and export8 value
int ref_grid_geom(void* h, int32_t* g4) {
  RefMap* m = static_cast<RefMap*>(h);
  if (!m->mapper) return -1;
  const OccGrid& G = m->mapper->grid();
  g4[0] = G.x0(); g4[1] = G.y0(); g4[2] = G.width(); g4[3] = G.height();
  return 0;
}
int ref_grid_cells(void* h, int16_t* L, uint8_t* seen, int8_t* c8) {
  RefMap* m = static_cast<RefMap*>(h);
  if (!m->mapper) return -1;
  const OccGrid& G = m->mapper->grid();
  const int w = G.width(), hh = G.height();
  std::vector<int8_t> e = G.export8();
  for (int y = 0; y < hh; ++y)
    for (int x = 0; x < w; ++x) {
      const size_t i = size_t(y) * w + x;
      const int ix = G.x0() + x, iy = G.y0() + y;
      if (L) L[i] = int16_t(std::lround(G.logOdds(ix, iy) * OccGrid::kQ));
      if (seen) seen[i] = G.seen(ix, iy);
      if (c8) c8[i] = e[i];
    }
  return w * hh;
}

// ---- standalone occupancy grid (config 3) ----
void* ref_occ_create(const float* grid5) {
  GridParams p;
  p.res = grid5[0]; p.l_hit = grid5[1]; p.l_miss = grid5[2]; p.l_min = grid5[3]; p.l_max = grid5[4];
  return new OccGrid(p);
}
void ref_occ_destroy(void* g) { delete static_cast<OccGrid*>(g); }
// laser hits (hx, hy), free-ray ends (fx, fy), match points (mx, my, mnx, mny) in the base frame
int ref_occ_insert(void* g, float ox, float oy, const float* hx, const float* hy, int nh, const float* fx, const float* fy, int nf,
                   const float* mx, const float* my, const float* mnx, const float* mny, int nm, const double* pose3) {
  Scan2 s;
  s.ox = ox; s.oy = oy;
  s.hx.assign(hx, hx + nh); s.hy.assign(hy, hy + nh);
  s.fx.assign(fx, fx + nf); s.fy.assign(fy, fy + nf);
  s.mx.assign(mx, mx + nm); s.my.assign(my, my + nm);
  if (mnx && mny) { s.mnx.assign(mnx, mnx + nm); s.mny.assign(mny, mny + nm); }
  return static_cast<OccGrid*>(g)->insert(s, Pose2{pose3[0], pose3[1], pose3[2]});
}
void ref_occ_geom(void* g, int32_t* g4) {
  const OccGrid& G = *static_cast<OccGrid*>(g);
  g4[0] = G.x0(); g4[1] = G.y0(); g4[2] = G.width(); g4[3] = G.height();
}
void ref_occ_cells(void* g, int16_t* L, uint8_t* seen, int8_t* c8, float* prob) {
  const OccGrid& G = *static_cast<OccGrid*>(g);
  std::vector<int8_t> e = G.export8();
  for (int y = 0; y < G.height(); ++y)
    for (int x = 0; x < G.width(); ++x) {
      const size_t i = size_t(y) * G.width() + x;
      const int ix = G.x0() + x, iy = G.y0() + y;
      if (L) L[i] = int16_t(std::lround(G.logOdds(ix, iy) * OccGrid::kQ));
      if (seen) seen[i] = G.seen(ix, iy);
      if (c8) c8[i] = e[i];
      if (prob) prob[i] = G.prob(ix, iy);
    }
}

// ---- makeScan on one depth frame (no body capsules, no attach filter) ----
// out sizes: returns nh, nf, nm in n3; arrays must hold 720 / 720 / 12288 entries.
int ref_make_scan(int w, int h, const float* depth, float fx, float fy, float cx, float cy, const float* T_bc, const float* eef_base6,
                  float* hx, float* hy, float* fxo, float* fyo, float* mx, float* my, float* mnx, float* mny, int16_t* sig, float sig_cell,
                  int32_t* n3, float* oxy) {
  DepthView dv;
  dv.w = w; dv.h = h; dv.m = depth;
  dv.step = std::max(1, int(std::lround(w / 160.0)));
  dv.fx = fx; dv.fy = fy; dv.cx = cx; dv.cy = cy;
  memcpy(dv.T_bc, T_bc, sizeof(dv.T_bc));
  BodyState b;
  for (int s = 0; s < 2; ++s) for (int k = 0; k < 3; ++k) b.eef[s][k] = eef_base6[3 * s + k];
  ScanParams p;
  Scan2 out;
  ScanWork W;
  makeScan(dv, b, p, &out, nullptr, nullptr, &W, sig_cell);
  n3[0] = int(out.hx.size()); n3[1] = int(out.fx.size()); n3[2] = int(out.mx.size());
  for (size_t k = 0; k < out.hx.size(); ++k) { hx[k] = out.hx[k]; hy[k] = out.hy[k]; }
  for (size_t k = 0; k < out.fx.size(); ++k) { fxo[k] = out.fx[k]; fyo[k] = out.fy[k]; }
  for (size_t k = 0; k < out.mx.size(); ++k) { mx[k] = out.mx[k]; my[k] = out.my[k]; mnx[k] = out.mnx[k]; mny[k] = out.mny[k]; }
  if (sig) for (size_t k = 0; k < out.sig.size(); ++k) sig[k] = out.sig[k];
  oxy[0] = out.ox; oxy[1] = out.oy;
  return 0;
}

// ---- objprob primitives (known-answer pins for the restatement and the kernels) ----
int ref_plane_fit(const float* xyz, int n, double tau, uint64_t seed, int max_iters, double* out /* ok,n0,n1,n2,thick,inl,zmed,zlo,zhi,hspan */) {
  const ApPlane p = apPlaneFit(xyz, n, tau, seed, max_iters);
  out[0] = p.ok; out[1] = p.n[0]; out[2] = p.n[1]; out[3] = p.n[2]; out[4] = p.thick; out[5] = p.inl; out[6] = p.zmed; out[7] = p.zlo;
  out[8] = p.zhi; out[9] = p.hspan;
  return p.ok;
}
uint64_t ref_ap_seed(uint64_t a, uint64_t b) { return apSeed(a, b); }
void ref_to_f16(const float* in, uint16_t* out, int n) { apToF16(in, out, n); }
uint64_t ref_voxel_key(float x, float y, float z, float inv) { return voxelKey(x, y, z, inv); }
double ref_contact(const float* cloud, int nc, const float* pts, int np, double cell) {
  ApContactIdx idx;
  apBuildContact(cloud, nc, cell, &idx);
  return apContact(pts, np, idx, cell);
}

// ---- text model: apLabelLogLik and apName (objprob.cpp:287-310, :396-455) ----
static ApText make_text(int dim, int n_labels, int rows, const float* text, const int32_t* row_label, float scale, float bias,
                        const float* log_prior, const float* ls_mu, const float* ls_sd, const int32_t* parent, int object_label) {
  ApText T;
  T.dim = dim;
  T.n_labels = n_labels;
  T.text.assign(text, text + size_t(rows) * dim);
  T.row_label.assign(row_label, row_label + rows);
  T.scale = scale;
  T.bias = bias;
  if (log_prior) T.log_prior.assign(log_prior, log_prior + n_labels);
  if (ls_mu && ls_sd) { T.ls_mu.assign(ls_mu, ls_mu + n_labels); T.ls_sd.assign(ls_sd, ls_sd + n_labels); }
  if (parent) T.parent.assign(parent, parent + n_labels);
  T.object_label = object_label;
  return T;
}

void ref_label_loglik(int dim, int n_labels, int rows, const float* text, const int32_t* row_label, float scale, float bias,
                      const float* z, int n, float* out) {
  const ApText T = make_text(dim, n_labels, rows, text, row_label, scale, bias, nullptr, nullptr, nullptr, nullptr, -1);
  std::vector<float> ll;
  for (int i = 0; i < n; ++i) {
    apLabelLogLik(T, z + size_t(i) * dim, &ll);
    for (int l = 0; l < n_labels; ++l) out[size_t(i) * n_labels + l] = ll[size_t(l)];
  }
}

// apName of one object; L arrays of n_labels (NULL = empty vector).  out: post[n_labels],
// f6 = {name_lab, name_p, top_lab, top_p, name_H, rolled}; returns 1 if apName produced a name.
int ref_name(int dim, int n_labels, int rows, const float* text, const int32_t* row_label, float scale, float bias,
             const float* log_prior, const float* ls_mu, const float* ls_sd, const int32_t* parent, int object_label,
             double whole_w, double name_wmax, double size_w, double name_tau, const float* L_frag, double lw_frag,
             const float* L_whole, double lw_whole, const float* L_ext, const float* L_geo, double size, float* post, double* f6) {
  const ApText T = make_text(dim, n_labels, rows, text, row_label, scale, bias, log_prior, ls_mu, ls_sd, parent, object_label);
  ApParams p;
  p.whole_w = whole_w; p.name_wmax = name_wmax; p.size_w = size_w; p.name_tau = name_tau;
  ApState s;
  if (L_frag) s.L_frag.assign(L_frag, L_frag + n_labels);
  if (L_whole) s.L_whole.assign(L_whole, L_whole + n_labels);
  if (L_ext) s.L_ext.assign(L_ext, L_ext + n_labels);
  if (L_geo) s.L_geo.assign(L_geo, L_geo + n_labels);
  s.lw_frag = lw_frag;
  s.lw_whole = lw_whole;
  apName(s, T, p, size);
  for (int l = 0; l < n_labels; ++l) post[l] = size_t(l) < s.post.size() ? s.post[size_t(l)] : 0.f;
  f6[0] = s.name_lab; f6[1] = s.name_p; f6[2] = s.top_lab; f6[3] = s.top_p; f6[4] = s.name_H; f6[5] = s.rolled;
  return !s.post.empty();
}

}  // extern "C"
