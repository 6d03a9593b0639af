// collide.hpp — swept-box traces and point-contents queries against BSP clip
// hulls (GoldSrc pmove collision: PM_RecursiveHullCheck, PM_HullPointContents,
// PM_PlayerTrace, PM_PointContents).
//
// All arithmetic is float32 in the same operation order as the engine so that
// a trace here returns bit-identical fractions/endpoints to the reference core
// (src/trace.c:12-236) on the same map. Build with -ffp-contract=off (host)
// or -fmad=false (device). Header-only: the host env and the GPU env compile
// the same functions (SURF_HD).
//
// The descent is the classic GoldSrc pmove hull check: split the segment
// at each node plane (nudged by DIST_EPSILON toward the near side), recurse into
// the near child, and if the far side of the split point is solid, report the
// split plane; if the split point itself lands in solid, back it off in 0.05
// steps of the parameter. Float expression order matters for parity and is
// kept identical to the engine's (reference: src/trace.c:26-119).
#pragma once
#include <cstring>

#include "map.hpp"

namespace surf {

struct Trace {
  bool allsolid = false, startsolid = false, inopen = false, inwater = false;
  float fraction = 1.f;
  float endpos[3] = {0, 0, 0};
  float normal[3] = {0, 0, 0};       // plane normal facing the motion
  float dist = 0;
  int ent = -1;                      // -1 none, 0 world, k>0 -> solids[k-1]
};

constexpr float kDistEpsilon = 0.03125f;

// Contents at point p (tree-local coordinates) starting at node `num`.
SURF_HD inline int hull_point_contents(const HullView& h, int num, const float p[3]);

// Trace a box (pmove usehull 0 stand, 1 duck, 2 point) through the world and
// every solid brush entity whose padded bounds overlap the move:
//   trace_player(const MapView&, int usehull, start, end, Trace*)
// Trace against one brush model only (point or player hull):
//   trace_model(const MapView&, int model, origin, usehull, start, end, Trace*)
// World hull-0 contents with currents folded into water, then contents volumes:
//   point_contents(const MapView&, p)
// True if a player with `usehull` at `origin` is inside trigger t's expanded hull:
//   trigger_contains(const MapView&, const Trigger&, usehull, origin)
// The Map overloads at the end forward to the view (host code).
namespace detail {

SURF_HD inline float dot3(const float* a, const float* b) { return a[0] * b[0] + a[1] * b[1] + a[2] * b[2]; }

SURF_HD inline float plane_side(const Plane& pl, const float* p) {
  return pl.type < 3 ? p[pl.type] - pl.dist : dot3(p, pl.normal) - pl.dist;
}

constexpr int kDescentDepthDevice = 64;   // device: local-memory continuation stack
constexpr int kDescentDepthHost = 512;
#if defined(__CUDA_ARCH__)
constexpr int kDescentDepth = kDescentDepthDevice;
#else
constexpr int kDescentDepth = kDescentDepthHost;
#endif

// The recursive descent written as a loop with an explicit stack of pending
// continuations (a CUDA thread has no deep call stack). Only the non-tail
// call (into the near child of a straddled node) pushes a frame; the tail
// calls reuse the current one. Every arithmetic expression is the recursive
// version's, so results are bit-identical. Returns false once an impact has
// been recorded. A tree deeper than the stack sets tr->allsolid (and
// startsolid), reported as a stuck trace; callers check tree depths up front.
struct HullDescent {
  const HullView& h;
  Trace* tr;

  struct Frame {
    int num, near;
    float f1, f2, s;
    float p1[3], p2[3];
  };

  // where a point query that would start at the root may start (HullGrid)
  SURF_HD int root_of(const float* p) const {
    const int32_t g = h.grid.point_start(p);
    return g != HullGrid::kNone ? g : h.first;
  }

  SURF_HD bool run(int num, float f1, float f2, const float* p1_in, const float* p2_in) {
    Frame stack[kDescentDepth];
    int sp = 0;
    float p1[3] = {p1_in[0], p1_in[1], p1_in[2]};
    float p2[3] = {p2_in[0], p2_in[1], p2_in[2]};
    bool ret = true, returning = false;
    for (;;) {
      if (!returning) {
        if (num < 0) {
          if (num == kSolid) {
            tr->startsolid = true;
          } else {
            tr->allsolid = false;
            if (num == kEmpty) tr->inopen = true; else tr->inwater = true;
          }
          ret = true;
          returning = true;
          continue;
        }
        if (h.first >= h.last) {            // empty tree
          tr->allsolid = false;
          tr->inopen = true;
          ret = true;
          returning = true;
          continue;
        }
        const Clipnode& node = h.nodes[num];
        const Plane& pl = h.planes[node.plane];
        float t1 = plane_side(pl, p1);
        float t2 = plane_side(pl, p2);
        if (t1 >= 0.f && t2 >= 0.f) { num = node.child[0]; continue; }
        float s;
        if (t1 >= 0.f) {
          s = t1 - kDistEpsilon;
        } else {
          if (t2 < 0.f) { num = node.child[1]; continue; }
          s = t1 + kDistEpsilon;
        }
        s = s / (t1 - t2);
        if (s >= 0.f) { if (s > 1.f) s = 1.f; } else { s = 0.f; }
        const float df = f2 - f1;
        float fmid = df * s + f1;
        float mid[3];
        for (int k = 0; k < 3; ++k) mid[k] = (p2[k] - p1[k]) * s + p1[k];
        const int near = t1 >= 0.f ? 0 : 1;
        if (sp == kDescentDepth) {          // deeper than any map this build accepts
          tr->allsolid = true;
          tr->startsolid = true;
          return false;
        }
        Frame& fr = stack[sp++];
        fr.num = num;
        fr.near = near;
        fr.f1 = f1;
        fr.f2 = f2;
        fr.s = s;
        for (int k = 0; k < 3; ++k) { fr.p1[k] = p1[k]; fr.p2[k] = p2[k]; }
        num = node.child[near];             // run(child[near], f1, fmid, p1, mid)
        f2 = fmid;
        for (int k = 0; k < 3; ++k) p2[k] = mid[k];
        continue;
      }
      // a call returned `ret` to the frame on top of the stack
      if (sp == 0) return ret;
      const Frame fr = stack[--sp];
      if (!ret) continue;                   // if (!run(near ...)) return false;
      const Clipnode& node = h.nodes[fr.num];
      const Plane& pl = h.planes[node.plane];
      const int near = fr.near;
      float s = fr.s;
      const float df = fr.f2 - fr.f1;
      float fmid = df * s + fr.f1;
      float mid[3];
      for (int k = 0; k < 3; ++k) mid[k] = (fr.p2[k] - fr.p1[k]) * s + fr.p1[k];
      if (hull_point_contents(h, node.child[near ^ 1], mid) != kSolid) {
        num = node.child[near ^ 1];         // return run(child[near ^ 1], fmid, f2, mid, p2);
        f1 = fmid;
        f2 = fr.f2;
        for (int k = 0; k < 3; ++k) { p1[k] = mid[k]; p2[k] = fr.p2[k]; }
        returning = false;
        continue;
      }
      ret = false;
      if (tr->allsolid) continue;
      if (near) {
        for (int k = 0; k < 3; ++k) tr->normal[k] = -pl.normal[k];
        tr->dist = -pl.dist;
      } else {
        for (int k = 0; k < 3; ++k) tr->normal[k] = pl.normal[k];
        tr->dist = pl.dist;
      }
      // Back the impact point off until it is outside solid (numeric safety).
      // A point query from the root may start at its grid cell's node.
      while (hull_point_contents(h, root_of(mid), mid) == kSolid) {
        s = static_cast<float>(s - 0.05);
        if (s < 0.f) break;
        fmid = df * s + fr.f1;
        for (int k = 0; k < 3; ++k) mid[k] = (fr.p2[k] - fr.p1[k]) * s + fr.p1[k];
      }
      tr->fraction = fmid;
      for (int k = 0; k < 3; ++k) tr->endpos[k] = mid[k];
    }
  }
};

// Depth of a clip tree below `num` (iterative; callers size the descent stack).
SURF_HD inline int hull_depth(const HullView& h, int num, int limit) {
  if (num < 0 || h.first >= h.last) return 0;
  int stack_n[256], stack_d[256];
  int sp = 0, best = 0;
  stack_n[sp] = num;
  stack_d[sp++] = 1;
  while (sp) {
    const int n = stack_n[--sp], d = stack_d[sp];
    if (d > best) best = d;
    if (best > limit) return best;
    const Clipnode& node = h.nodes[n];
    for (int c = 0; c < 2; ++c)
      if (node.child[c] >= 0 && sp < 256) { stack_n[sp] = node.child[c]; stack_d[sp++] = d + 1; }
  }
  return best;
}

// Sweep one brush model; mirrors the per-entity body of PM_PlayerTrace.
SURF_HD SURF_HD_NOINLINE void clip_model(const MapView& m, int model, const float ent_origin[3], int usehull, const float start[3],
                const float end[3], Trace* out) {
  HullView h = m.hull(model, bsp_hull_of_usehull(usehull));
  float off[3], a[3], b[3];
  for (int k = 0; k < 3; ++k) {
    off[k] = h.clip_mins[k] - player_mins(usehull, k) + ent_origin[k];
    a[k] = start[k] - off[k];
    b[k] = end[k] - off[k];
  }
  *out = Trace();
  out->allsolid = true;
  out->fraction = 1.f;
  for (int k = 0; k < 3; ++k) out->endpos[k] = end[k];
  // both endpoints in cells of the same start node: the descent from the
  // root would reach it without a split (HullGrid), so start there
  const int32_t g0 = h.grid.segment_start(a, b);
  const int node0 = g0 != HullGrid::kNone ? g0 : h.first;
  HullDescent d{h, out};
  d.run(node0, 0.f, 1.f, a, b);
  if (out->allsolid) out->startsolid = true;
  if (out->startsolid) out->fraction = 0.f;
  if (out->fraction != 1.f)
    for (int k = 0; k < 3; ++k) out->endpos[k] = (end[k] - start[k]) * out->fraction + start[k];
}

}  // namespace detail

SURF_HD inline int hull_point_contents(const HullView& h, int num, const float p[3]) {
  if (h.first >= h.last) return kEmpty;
  while (num >= 0) {
    const Clipnode& node = h.nodes[num];
    num = detail::plane_side(h.planes[node.plane], p) >= 0.f ? node.child[0] : node.child[1];
  }
  return num;
}

SURF_HD inline void trace_model(const MapView& m, int model, const float origin[3], int usehull, const float start[3],
                 const float end[3], Trace* tr) {
  detail::clip_model(m, model, origin, usehull, start, end, tr);
  tr->ent = 0;
}

SURF_HD inline void trace_player(const MapView& m, int usehull, const float start[3], const float end[3], Trace* tr) {
  Trace t;
  detail::clip_model(m, 0, m.models[0].origin, usehull, start, end, &t);
  *tr = t;
  tr->ent = (t.fraction == 1.f && !t.startsolid) ? -1 : 0;
  const float pad = 40.f;                 // broad-phase margin >= largest hull half-extent
  float lo[3], hi[3];
  for (int k = 0; k < 3; ++k) {
    lo[k] = (start[k] < end[k] ? start[k] : end[k]) - pad;
    hi[k] = (start[k] > end[k] ? start[k] : end[k]) + pad;
  }
  for (int i = 0; i < m.solids.size(); ++i) {
    const BrushEntity& s = m.solids[i];
    if (lo[0] > s.absmax[0] || hi[0] < s.absmin[0] || lo[1] > s.absmax[1] || hi[1] < s.absmin[1] ||
        lo[2] > s.absmax[2] || hi[2] < s.absmin[2])
      continue;
    detail::clip_model(m, s.model, s.origin, usehull, start, end, &t);
    if (t.fraction < tr->fraction) {
      *tr = t;
      tr->ent = i + 1;
    }
  }
}

namespace detail {
// Whether the expanded hull of `model` holds the player box (usehull) at p:
// the startsolid of clip_model(model, ent_origin, usehull, p, p). A segment of
// zero length never straddles a plane (both ends give the same plane_side),
// so the descent visits one child per node down to a single leaf, and only a
// solid leaf makes it start solid. Same offsets, start node and node tests
// as clip_model, so the answer is the same bit for bit (p must not be NaN:
// a NaN side takes clip_model's split branch).
SURF_HD inline bool model_point_solid(const MapView& m, int model, const float ent_origin[3], int usehull,
                                      const float p[3]) {
  HullView h = m.hull(model, bsp_hull_of_usehull(usehull));
  float a[3];
  for (int k = 0; k < 3; ++k) {
    const float off = h.clip_mins[k] - player_mins(usehull, k) + ent_origin[k];
    a[k] = p[k] - off;
  }
  const int32_t g = h.grid.point_start(a);        // segment_start(a, a) picks the same node
  int num = g != HullGrid::kNone ? g : h.first;
  if (num >= 0 && h.first >= h.last) return false;   // empty tree: in the open
  while (num >= 0) {
    const Clipnode& node = h.nodes[num];
    num = plane_side(h.planes[node.plane], a) >= 0.f ? node.child[0] : node.child[1];
  }
  return num == kSolid;
}
}  // namespace detail

// trace_player(m, usehull, p, p).startsolid without the sweep: the world or any
// solid brush entity whose padded bounds hold p puts p in solid (a model that
// starts solid reports fraction 0, which no later model can undercut). This is
// the engine's PM_TestPlayerPosition question (stuck checks, unduck headroom),
// asked once or twice per tick, so it skips the segment set-up and the
// descent's continuation stack.
SURF_HD inline bool player_point_solid(const MapView& m, int usehull, const float p[3]) {
  if (p[0] != p[0] || p[1] != p[1] || p[2] != p[2]) {
    Trace tr;
    trace_player(m, usehull, p, p, &tr);
    return tr.startsolid;
  }
  if (detail::model_point_solid(m, 0, m.models[0].origin, usehull, p)) return true;
  const float pad = 40.f;                 // trace_player's broad-phase margin
  for (int i = 0; i < m.solids.size(); ++i) {
    const BrushEntity& s = m.solids[i];
    if (p[0] - pad > s.absmax[0] || p[0] + pad < s.absmin[0] || p[1] - pad > s.absmax[1] ||
        p[1] + pad < s.absmin[1] || p[2] - pad > s.absmax[2] || p[2] + pad < s.absmin[2])
      continue;
    if (detail::model_point_solid(m, s.model, s.origin, usehull, p)) return true;
  }
  return false;
}

SURF_HD inline int point_contents(const MapView& m, const float p[3]) {
  HullView h0 = m.hull(0, 0);
  const int32_t g = h0.grid.point_start(p);
  int c = hull_point_contents(h0, g != HullGrid::kNone ? g : h0.first, p);
  if (c <= kCurrent0 && c >= kCurrentDown) c = kWater;
  else if (c == kSolid) return kSolid;
  for (const BrushEntity& v : m.volumes) {
    if (v.contents == kEmpty) continue;
    if (p[0] < v.absmin[0] || p[0] > v.absmax[0] || p[1] < v.absmin[1] || p[1] > v.absmax[1] ||
        p[2] < v.absmin[2] || p[2] > v.absmax[2])
      continue;
    float local[3] = {p[0] - v.origin[0], p[1] - v.origin[1], p[2] - v.origin[2]};
    HullView vh = m.hull(v.model, 0);
    if (hull_point_contents(vh, vh.first, local) != kEmpty) return v.contents;
  }
  return c;
}

SURF_HD inline bool trigger_contains(const MapView& m, const Trigger& t, int usehull, const float origin[3]) {
  HullView h = m.hull(t.model, bsp_hull_of_usehull(usehull));
  float local[3];
  for (int k = 0; k < 3; ++k) local[k] = origin[k] - (h.clip_mins[k] - player_mins(usehull, k) + t.origin[k]);
  return hull_point_contents(h, h.first, local) == kSolid;
}

inline void trace_player(const Map& m, int usehull, const float start[3], const float end[3], Trace* tr) {
  trace_player(m.view(), usehull, start, end, tr);
}
inline void trace_model(const Map& m, int model, const float origin[3], int usehull, const float start[3],
                        const float end[3], Trace* tr) {
  trace_model(m.view(), model, origin, usehull, start, end, tr);
}
inline int point_contents(const Map& m, const float p[3]) { return point_contents(m.view(), p); }
inline bool trigger_contains(const Map& m, const Trigger& t, int usehull, const float origin[3]) {
  return trigger_contains(m.view(), t, usehull, origin);
}

}  // namespace surf
