// collide.hpp — swept-box traces and point-contents queries against BSP clip
// hulls (GoldSrc pmove collision: PM_RecursiveHullCheck, PM_HullPointContents,
// PM_PlayerTrace, PM_PointContents).
//
// All arithmetic is float32 in the same operation order as the engine so that
// a trace here returns bit-identical fractions/endpoints to the reference core
// (src/trace.c:12-236) on the same map. Build with -ffp-contract=off.
#pragma once
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
int hull_point_contents(const HullView& h, int num, const float p[3]);

// Trace a box (pmove usehull 0 stand, 1 duck, 2 point) through the world and
// every solid brush entity whose padded bounds overlap the move.
void trace_player(const Map& m, int usehull, const float start[3], const float end[3], Trace* tr);

// Trace against one brush model only (point or player hull).
void trace_model(const Map& m, int model, const float origin[3], int usehull, const float start[3],
                 const float end[3], Trace* tr);

// World hull-0 contents with currents folded into water, then contents volumes.
int point_contents(const Map& m, const float p[3]);

// True if a player with `usehull` at `origin` is inside trigger t's expanded hull.
bool trigger_contains(const Map& m, const Trigger& t, int usehull, const float origin[3]);

}  // namespace surf
