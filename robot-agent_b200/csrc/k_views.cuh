// Best views and cloud colours of a keyframe: the RGB side of the reference's keyframe glue
// (scenemap src/capi.cpp:903-998, include/scenemap/bestview.hpp, src/bestview.cpp).
//
// After ObjectMap::update, the glue
//   1. sets the quality of the view of every object named by a new "moved" (2) or "put down" (5)
//      event to 0, so that the next observation replaces it (capi.cpp:903-909);
//   2. drops the views of objects that no longer exist (:910-914);
//   3. makes every detection attached to an object a candidate when its quality
//      q = valid mask area x score is >= the object's view quality, and its crop box
//      (cropGeometry: detection box + 10 % per side, clipped, longer side <= 256) is not empty
//      (:915-943);
//   4. colours the observation cloud points from the RGBA image (gatherRgbHost, :945-956), crops
//      the candidates (cropRgbHost area average, cropDepthMm nearest, cropMask) (:958-972), and
//      installs them in detection order, each one unless its quality is below the view it would
//      replace, with version = ++view counter (:985-998).
// Here the view quality lives with the object record (ObjRec::view_q / has_view: a view of a
// dead object goes with the record, step 2), k_views_pick runs steps 1 and 3 and the install
// decisions, k_views_crop crops the installed views into per-detection image slots, and
// k_cloud_add colours the points (gather_rgba in cloud_add).  The images leave the device
// through smg_get_views: the caller keeps them, as the reference's context keeps its views map.
#pragma once
#include "k_assoc.cuh"
#include "k_cloud.cuh"

#define VIEW_MARGIN 0.10f   // kCropMargin (capi.cpp:87)
#define VIEW_THREADS 128
#define VCROP_THREADS 256

// cropGeometry (bestview.cpp:9-22): float margins, floor / ceil, clip to the image, then the
// output size lround(side * min(1, max_side / longer side)), at least 1.
DEV bool crop_geometry(const float* b, int img_w, int img_h, float margin, int max_side, int* box, int* ow, int* oh) {
  const float mx = margin * (b[2] - b[0]), my = margin * (b[3] - b[1]);
  box[0] = vclampi((int)floorf(b[0] - mx), 0, img_w);
  box[1] = vclampi((int)floorf(b[1] - my), 0, img_h);
  box[2] = vclampi((int)ceilf(b[2] + mx), 0, img_w);
  box[3] = vclampi((int)ceilf(b[3] + my), 0, img_h);
  const int bw = box[2] - box[0], bh = box[3] - box[1];
  if (bw <= 0 || bh <= 0) return false;
  const double r = (double)max_side / (double)(bw > bh ? bw : bh);
  const double s = r < 1.0 ? r : 1.0;
  const long lw = lround((double)bw * s), lh = lround((double)bh * s);
  *ow = lw > 1 ? (int)lw : 1;
  *oh = lh > 1 ? (int)lh : 1;
  return true;
}

// Slot of the object with this id in map m, or -1.  All threads of the block call it.
DEV int view_find_slot(const Batch& B, int m, uint32_t id, int* sh) {
  if (threadIdx.x == 0) *sh = -1;
  __syncthreads();
  const int n = B.maps[m].n_obj;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int s = slot_at(B, m, i);
    if (INB(s, B.O, 901) && B.objs[oglob(B, m, s)].id == id) *sh = s;   // ids are unique
  }
  __syncthreads();
  const int r = *sh;
  __syncthreads();
  return r;
}

// Steps 1 and 3 and the install decisions, one CTA per map.  Pass A applies the candidate test
// to every detection against the views as step 1 left them (capi.cpp:921-922); pass B installs
// the candidates in detection order, each unless its quality is below the view as the installs
// before it left it (capi.cpp:994-996); the object records take the final view quality last.
__global__ void __launch_bounds__(VIEW_THREADS) k_views_pick(Batch B) {
  __shared__ int sh_slot;
  __shared__ int vslot[SMG_MAX_DET];        // object slot of detection k's object, -1 = none
  __shared__ uint32_t acc_id[SMG_MAX_DET];  // views installed so far this keyframe
  __shared__ double acc_q[SMG_MAX_DET];
  __shared__ int acc_k[SMG_MAX_DET];
  const int m = B.map0 + blockIdx.x, tid = threadIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active) return;
  MapRec* R = &B.maps[m];
  // 1. moved / put-down events of this keyframe reset the quality of the object's view (every
  // keyframe, with or without an image: views picked earlier may exist)
  const int ne = min(R->n_events, SMG_MAX_EVENTS);
  for (int e = 0; e < ne; ++e) {
    const EventRec ev = B.events[(size_t)m * SMG_MAX_EVENTS + e];
    if (ev.kind != 2 && ev.kind != 5) continue;
    const int s = view_find_slot(B, m, ev.id, &sh_slot);
    if (tid == 0 && s >= 0) B.objs[oglob(B, m, s)].view_q = 0.0;
    __syncthreads();
  }
  if (!F.views_on) {
    if (tid == 0) R->n_vnew = 0;
    return;
  }
  const int nd = min(F.n_det, B.max_det);
  for (int k = 0; k < nd; ++k) {
    const uint32_t id = B.assoc[(size_t)m * B.max_det + k].obj_id;
    const int s = id ? view_find_slot(B, m, id, &sh_slot) : -1;
    if (tid == 0) vslot[k] = s;
  }
  __syncthreads();
  if (tid != 0) return;
  // A. candidates (a dead object has no view: step 2)
  for (int k = 0; k < nd; ++k) {
    const AssocRec a = B.assoc[(size_t)m * B.max_det + k];
    ViewRec& V = B.vrec[(size_t)m * B.max_det + k];
    V.cand = 0;
    V.final_ = 0;
    if (!a.obj_id) continue;
    const ObjRec* o = vslot[k] >= 0 ? &B.objs[oglob(B, m, vslot[k])] : nullptr;
    const float sc = F.score[k];
    const double q = (double)a.area_px * (double)sc;
    if (o && o->has_view && q < o->view_q) continue;
    int box[4], ow, oh;
    if (!crop_geometry(F.box[k], F.img_w, F.img_h, VIEW_MARGIN, SMG_VIEW_MAX_SIDE, box, &ow, &oh)) continue;
    V.cand = 1;
    V.id = a.obj_id;
    V.q = q;
    V.stamp = F.stamp;
    for (int c = 0; c < 4; ++c) { V.box[c] = box[c]; V.det_box[c] = (int32_t)lroundf(F.box[k][c]); }
    V.mask_area = a.area_px;
    V.depth_m = a.depth_med;
    V.score = sc;
    for (int c = 0; c < 12; ++c) V.cam_T[c] = F.T_mc[c];
    V.w = ow;
    V.h = oh;
  }
  // B. installs, detection order
  int n_acc = 0;
  for (int k = 0; k < nd; ++k) {
    ViewRec& V = B.vrec[(size_t)m * B.max_det + k];
    if (!V.cand) continue;
    int last = -1;
    for (int i = 0; i < n_acc; ++i)
      if (acc_id[i] == V.id) last = i;
    const ObjRec* o = vslot[k] >= 0 ? &B.objs[oglob(B, m, vslot[k])] : nullptr;
    const bool has_now = last >= 0 || (o && o->has_view);
    const double q_now = last >= 0 ? acc_q[last] : (o ? o->view_q : 0.0);
    if (has_now && V.q < q_now) continue;
    V.final_ = 1;
    V.version = ++R->view_ver;
    if (last >= 0) B.vrec[(size_t)m * B.max_det + acc_k[last]].final_ = 0;
    acc_id[n_acc] = V.id;
    acc_q[n_acc] = V.q;
    acc_k[n_acc] = k;
    ++n_acc;
  }
  int n = 0;
  for (int k = 0; k < nd; ++k) {
    const ViewRec& V = B.vrec[(size_t)m * B.max_det + k];
    if (!V.final_) continue;
    R->vnew[n++] = k;
    if (vslot[k] >= 0) {
      ObjRec& o = B.objs[oglob(B, m, vslot[k])];
      o.has_view = 1;
      o.view_q = V.q;
    }
  }
  R->n_vnew = n;
}

// Step 4 for the installed views: one CTA per (detection, map) whose view was installed,
// writing the crop into that detection's image slots (rgb w x h x 3, depth w x h uint16 mm,
// mask w x h), rows packed to the crop's width.
__global__ void __launch_bounds__(VCROP_THREADS) k_views_crop(Batch B) {
  const int m = B.map0 + blockIdx.y, k = blockIdx.x;
  const FrameDev& F = B.frames[m];
  if (!F.active || !F.views_on || k >= min(F.n_det, B.max_det)) return;
  const ViewRec& V = B.vrec[(size_t)m * B.max_det + k];
  if (!V.final_) return;
  const size_t vs = (size_t)m * B.max_det + k;
  uint8_t* orgb = B.vrgb + vs * VIEW_PIX * 3;
  uint16_t* odep = B.vdepth + vs * VIEW_PIX;
  uint8_t* omsk = B.vmask + vs * VIEW_PIX;
  const int ow = V.w, oh = V.h, x0 = V.box[0], y0 = V.box[1];
  const int bw = V.box[2] - V.box[0], bh = V.box[3] - V.box[1];
  if (!INB(ow * oh - 1, VIEW_PIX, 902)) return;
  const int W = F.w, H = F.h;
  const float* dsrc = F.depth_host ? F.depth_host : F.depth;   // a host frame read in place
  const uint16_t* lsrc = F.label_host ? F.label_host : F.label;
  const bool bits_form = F.mask_bits != nullptr;
  const uint32_t* bits = bits_form ? F.mask_bits + (size_t)k * F.mask_words : nullptr;
  const uint16_t L = F.det_label[k];
  // depth: same box, scaled by depth size / detector size (1 here: the sizes agree)
  const double sx = F.img_w > 0 ? (double)W / F.img_w : 1.0, sy = F.img_h > 0 ? (double)H / F.img_h : 1.0;
  const double dbw = (double)bw, dbh = (double)bh;
  for (int p = threadIdx.x; p < ow * oh; p += blockDim.x) {
    const int j = p / ow, i = p - j * ow;
    // cropRgbHost (bestview.cpp:25-43): output pixel (i, j) averages source pixels
    // [x0 + i*bw/ow, max(that + 1, x0 + (i+1)*bw/ow)) x the same in y, rounded to nearest
    {
      const int ya = y0 + j * bh / oh, yb = max(ya + 1, y0 + (j + 1) * bh / oh);
      const int xa = x0 + i * bw / ow, xb = max(xa + 1, x0 + (i + 1) * bw / ow);
      uint32_t s0 = 0, s1 = 0, s2 = 0;
      for (int y = ya; y < yb; ++y) {
        if (!INB(y, H, 903)) break;
        const uchar4* row = (const uchar4*)(F.rgba + (size_t)y * W * 4);
        for (int x = xa; x < xb; ++x) {
          if (!INB(x, W, 904)) break;
          const uchar4 c = row[x];
          s0 += c.x; s1 += c.y; s2 += c.z;
        }
      }
      const uint32_t n = (uint32_t)((yb - ya) * (xb - xa));
      orgb[3 * p] = (uint8_t)((s0 + n / 2) / n);
      orgb[3 * p + 1] = (uint8_t)((s1 + n / 2) / n);
      orgb[3 * p + 2] = (uint8_t)((s2 + n / 2) / n);
    }
    // cropDepthMm (bestview.cpp:45-56): the pixel under the output pixel's centre, mm
    {
      const int v = vclampi((int)(((double)V.box[1] + ((double)j + 0.5) * dbh / (double)oh) * sy), 0, H - 1);
      const int u = vclampi((int)(((double)V.box[0] + ((double)i + 0.5) * dbw / (double)ow) * sx), 0, W - 1);
      const float z = dsrc[(size_t)v * W + u];
      odep[p] = (z > 0.f && z < 65.535f) ? (uint16_t)lroundf(z * 1000.f) : (uint16_t)0;
    }
    // cropMask (bestview.cpp:58-75): the mask cell under the output pixel's centre
    {
      uint8_t mv = 0;
      const double y = (double)V.box[1] + ((double)j + 0.5) * dbh / (double)oh;
      const double x = (double)V.box[0] + ((double)i + 0.5) * dbw / (double)ow;
      const int mj = (int)floor((y - (double)F.mask_oy) / (double)F.mask_sy);
      const int mi = (int)floor((x - (double)F.mask_ox) / (double)F.mask_sx);
      if (mj >= 0 && mj < F.mask_h && mi >= 0 && mi < F.mask_w) {
        const size_t c = (size_t)mj * F.mask_w + mi;
        if (bits_form) mv = ((bits[c >> 5] >> (c & 31)) & 1u) ? 255 : 0;
        else mv = lsrc[c] == L ? 255 : 0;   // label image: mask cell = pixel
      }
      omsk[p] = mv;
    }
  }
}
