// movement.hpp — Counter-Strike 1.6 player movement (pm_shared) over a Map.
//
// One call to PlayerMove::tick advances one player by one usercmd. The state
// layout is byte-compatible with the reference core's SurfState (108 bytes,
// src/surfcore.h:118-140) so state rows can be exchanged with it, recorded and
// restored. Precision discipline follows the published movement code: vec3
// storage is float, a handful of intermediate values are double ("real_t"),
// and every such site is marked where it happens.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

#include "collide.hpp"

namespace surf {

constexpr int kInJump = 2;       // usercmd button bits (HLSDK in_buttons.h)
constexpr int kInDuck = 4;
constexpr int kInForward = 1 << 3;
constexpr int kInBack = 1 << 4;
constexpr int kInMoveLeft = 1 << 9;
constexpr int kInMoveRight = 1 << 10;

struct Physics {                  // server cvars (SurfPhys-compatible, 60 bytes)
  float gravity = 800, airaccelerate = 100, accelerate = 5, friction = 4, edgefriction = 2;
  float stopspeed = 75, maxspeed = 320, player_maxspeed = 250, maxvelocity = 2000;
  float stepsize = 18, bounce = 1;
  int32_t msec = 10, enable_stamina = 1, enable_bhop_cap = 1, enable_duck = 1;
};
static_assert(sizeof(Physics) == 60, "Physics layout");

struct PlayerState {              // SurfState-compatible (108 bytes)
  float origin[3], velocity[3], basevelocity[3];
  float yaw, pitch;               // degrees; pitch is view-only (+ = up)
  float fuser2;                   // stamina countdown (ms)
  int32_t base_vel_flag, onground, oldbuttons, ducked, tick, seg_hint;
  float progress, best_progress;
  int32_t stuck_ticks, induck;
  float duck_time, waterjumptime;
  float movedir[3];
};
static_assert(sizeof(PlayerState) == 108, "PlayerState layout");

struct StuckMemo { int32_t index = 0; int32_t last_tick = 0; };   // CheckStuck bookkeeping

// Host-side cache of one player's last CategorizePosition down-trace. The
// trace is a pure function of the (static) map, the hull and the start point,
// so a player whose origin did not change between two categorisations (the
// end of one tick and the start of the next, while airborne) reuses it; the
// key is the origin's bit pattern. Nothing needs resetting: a hit returns
// exactly what the trace would.
struct GroundMemo {
  uint32_t key[3] = {0, 0, 0};
  int32_t hull = -1;
  Trace tr;
};

struct MoveResult { int waterlevel = 0; bool blocked = false; };

// Host and device: holds the map view and the physics settings by value, so
// a copy can be handed to a CUDA kernel as a parameter.
class PlayerMove {
 public:
  PlayerMove() = default;
  PlayerMove(const MapView& map, const Physics& phys) : map_(map), ph_(phys) {}
  PlayerMove(const Map& map, const Physics& phys) : map_(map.view()), ph_(phys) {}
  // yaw/pitch in GoldSrc convention (pitch + = down); fmove/smove in units.
  SURF_HD MoveResult tick(PlayerState* st, StuckMemo* memo, float yaw, float pitch, float fmove, float smove,
                          int buttons, int msec, GroundMemo* ground = nullptr) const;

 private:
  MapView map_;
  Physics ph_;
};

// The 54 nudge offsets of PM_CreateStuckTable, in engine order (host table).
const float (*stuck_offsets())[3];


// ---- implementation (header-only: the host env and the GPU env compile the
// same functions). Every function below states the movement rule it
// implements; the float / double mix at each arithmetic site is deliberate and
// must not be "cleaned up": it is what makes trajectories bit-identical to the
// engine and to the reference core (src/pm.c:51-975, spec
// docs/01-physics-spec.md:229-236).
namespace mv {

constexpr double kPi = 3.14159265358979323846;
constexpr float kBhopFactor = 1.2f;
constexpr float kViewStand = 17.0f, kViewDuck = 12.0f;
constexpr double kTimeToDuck = 0.4;
constexpr double kDuckSpeedMult = 0.333;
constexpr int kCrouchStuckSteps = 36;
constexpr int kMaxClimbSpeed = 200;
constexpr int kWaterJumpHeight = 8;
constexpr double kStopEpsilon = 0.1;
constexpr int kMaxClipPlanes = 5;

// --- vector helpers with the engine's precision at each site --------------
SURF_HD inline double dot_d(const float* a, const float* b) {     // float sum, widened on return
  float s = a[0] * b[0] + a[1] * b[1] + a[2] * b[2];
  return static_cast<double>(s);
}
SURF_HD inline double length_d(const float* v) {                  // float squares, double accumulator
  double acc = 0.0f;
  for (int i = 0; i < 3; ++i) acc += v[i] * v[i];
  return std::sqrt(acc);
}
SURF_HD inline double normalize(float* v) {                       // float radicand, double scale
  double len = std::sqrt(static_cast<double>(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]));
  if (len != 0.0) {
    double inv = 1.0 / len;
    v[0] = static_cast<float>(v[0] * inv);
    v[1] = static_cast<float>(v[1] * inv);
    v[2] = static_cast<float>(v[2] * inv);
  }
  return len;
}
SURF_HD inline bool nan_bits(float x) {                           // exponent all-ones
  int32_t b;
  memcpy(&b, &x, 4);
  return (b & (255 << 23)) == (255 << 23);
}
SURF_HD inline void copy3(float* d, const float* s) { d[0] = s[0]; d[1] = s[1]; d[2] = s[2]; }
SURF_HD inline void zero3(float* d) { d[0] = d[1] = d[2] = 0.0f; }

// AngleVectors: trig in double, most results rounded to float immediately,
// except cos(yaw) which stays double (it is a real_t local in the source).
SURF_HD inline void angle_vectors(const float* ang, float* fwd, float* right, float* up) {
  float sr, sp, sy, cr, cp;
  double cy, a;
  a = static_cast<double>(ang[1] * (kPi * 2 / 360));
  sy = static_cast<float>(std::sin(a));
  cy = std::cos(a);
  a = static_cast<double>(ang[0] * (kPi * 2 / 360));
  sp = static_cast<float>(std::sin(a));
  cp = static_cast<float>(std::cos(a));
  a = static_cast<double>(ang[2] * (kPi * 2 / 360));
  sr = static_cast<float>(std::sin(a));
  cr = static_cast<float>(std::cos(a));
  if (fwd) {
    fwd[0] = static_cast<float>(cp * cy);
    fwd[1] = cp * sy;
    fwd[2] = -sp;
  }
  if (right) {
    right[0] = static_cast<float>(-1 * sr * sp * cy + -1 * cr * -sy);
    right[1] = static_cast<float>(-1 * sr * sp * sy + -1 * cr * cy);
    right[2] = -1 * sr * cp;
  }
  if (up) {
    up[0] = static_cast<float>(cr * sp * cy + -sr * -sy);
    up[1] = static_cast<float>(cr * sp * sy + -sr * cy);
    up[2] = cr * cp;
  }
}

// ClipVelocity: remove the normal component (times overbounce); tiny results snap to 0.
SURF_HD inline int clip_velocity(const float* in, const float* n, float* out, float overbounce) {
  double nz = n[2];
  int blocked = 0;
  if (nz > 0) blocked |= 1;
  if (!nz) blocked |= 2;
  float back_f = (in[0] * n[0] + in[1] * n[1] + in[2] * n[2]) * overbounce;
  double back = back_f;
  for (int i = 0; i < 3; ++i) {
    float c = static_cast<float>(in[i] - n[i] * back);
    out[i] = c;
    if (out[i] > -kStopEpsilon && out[i] < kStopEpsilon) out[i] = 0;
  }
  return blocked;
}

// The 54 nudge offsets of PM_CreateStuckTable in engine order (the table the
// engine builds with float loop counters; every value is exact in binary).
SURF_HD inline float stuck_offset(int i, int k) {
  const float t[54][3] = {
      {0.0f, 0.0f, -0.125f}, {0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.125f}, {0.0f, -0.125f, 0.0f}, {0.0f, 0.0f, 0.0f}, {0.0f, 0.125f, 0.0f},
      {-0.125f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f}, {0.125f, 0.0f, 0.0f}, {-0.125f, -0.125f, -0.125f}, {-0.125f, -0.125f, 0.125f}, {-0.125f, 0.125f, -0.125f},
      {-0.125f, 0.125f, 0.125f}, {0.125f, -0.125f, -0.125f}, {0.125f, -0.125f, 0.125f}, {0.125f, 0.125f, -0.125f}, {0.125f, 0.125f, 0.125f}, {0.0f, 0.0f, 0.0f},
      {0.0f, 0.0f, 1.0f}, {0.0f, 0.0f, 6.0f}, {0.0f, -2.0f, 0.0f}, {0.0f, 0.0f, 0.0f}, {0.0f, 2.0f, 0.0f}, {-2.0f, 0.0f, 0.0f},
      {0.0f, 0.0f, 0.0f}, {2.0f, 0.0f, 0.0f}, {-2.0f, -2.0f, 0.0f}, {-2.0f, 0.0f, 0.0f}, {-2.0f, 2.0f, 0.0f}, {0.0f, -2.0f, 0.0f},
      {0.0f, 0.0f, 0.0f}, {0.0f, 2.0f, 0.0f}, {2.0f, -2.0f, 0.0f}, {2.0f, 0.0f, 0.0f}, {2.0f, 2.0f, 0.0f}, {-2.0f, -2.0f, 1.0f},
      {-2.0f, 0.0f, 1.0f}, {-2.0f, 2.0f, 1.0f}, {0.0f, -2.0f, 1.0f}, {0.0f, 0.0f, 1.0f}, {0.0f, 2.0f, 1.0f}, {2.0f, -2.0f, 1.0f},
      {2.0f, 0.0f, 1.0f}, {2.0f, 2.0f, 1.0f}, {-2.0f, -2.0f, 6.0f}, {-2.0f, 0.0f, 6.0f}, {-2.0f, 2.0f, 6.0f}, {0.0f, -2.0f, 6.0f},
      {0.0f, 0.0f, 6.0f}, {0.0f, 2.0f, 6.0f}, {2.0f, -2.0f, 6.0f}, {2.0f, 0.0f, 6.0f}, {2.0f, 2.0f, 6.0f}, {0.0f, 0.0f, 0.0f}};
  return t[i][k];
}

enum MoveType { kWalk = 0, kFly = 1 };

// Per-tick working set (pmove globals of the engine).
struct Mover {
  const MapView& map;
  const Physics& ph;
  PlayerState* st;
  StuckMemo* memo;
  GroundMemo* ground = nullptr;       // host only (null: always trace)
  float frametime = 0, maxspeed = 0, pfriction = 1.0f;
  float angles[3] = {0, 0, 0};
  float forward[3], right[3], up[3];
  float fmove = 0, smove = 0, upmove = 0;
  int buttons = 0, msec = 0, usehull = 0;
  int waterlevel = 0, watertype = kEmpty;
  float view_ofs = kViewStand;
  bool blocked_solid = false;

  SURF_HD void trace(int hull, const float* a, const float* b, Trace* tr) const { trace_player(map, hull, a, b, tr); }
  SURF_HD bool position_free(const float* p) const { return !player_point_solid(map, usehull, p); }

  // CheckVelocity: NaN scrub and per-axis clamp to sv_maxvelocity.
  SURF_HD void check_velocity() {
    for (int i = 0; i < 3; ++i) {
      if (nan_bits(st->velocity[i])) st->velocity[i] = 0;
      if (nan_bits(st->origin[i])) st->origin[i] = 0;
      if (st->velocity[i] > ph.maxvelocity) st->velocity[i] = ph.maxvelocity;
      else if (st->velocity[i] < -ph.maxvelocity) st->velocity[i] = -ph.maxvelocity;
    }
  }
  // Half of this frame's gravity before the move (double subtraction, one rounding).
  SURF_HD void add_gravity() {
    if (st->waterjumptime) return;
    double g = 1.0f;
    st->velocity[2] = static_cast<float>(st->velocity[2] - g * ph.gravity * 0.5f * frametime);
    st->velocity[2] += st->basevelocity[2] * frametime;
    st->basevelocity[2] = 0;
    check_velocity();
  }
  // The other half after the move ((gravity*frametime) is a float product).
  SURF_HD void fixup_gravity() {
    if (st->waterjumptime) return;
    double g = 1.0;
    st->velocity[2] = static_cast<float>(st->velocity[2] - static_cast<double>(ph.gravity * frametime) * g * 0.5);
    check_velocity();
  }
  // Ground friction with the edge-friction probe 16u ahead, 34u down.
  SURF_HD void friction() {
    if (st->waterjumptime) return;
    float* v = st->velocity;
    float speed = static_cast<float>(std::sqrt(static_cast<double>(v[0] * v[0] + v[1] * v[1] + v[2] * v[2])));
    if (speed < 0.1f) return;
    double drop = 0, fric, control, ns;
    if (st->onground != -1) {
      float a[3], b[3];
      Trace tr;
      a[0] = b[0] = st->origin[0] + v[0] / speed * 16;
      a[1] = b[1] = st->origin[1] + v[1] / speed * 16;
      a[2] = st->origin[2] + player_mins(usehull, 2);
      b[2] = a[2] - 34;
      trace(usehull, a, b, &tr);
      fric = tr.fraction == 1.0f ? ph.friction * ph.edgefriction : ph.friction;
      fric *= pfriction;
      control = speed < ph.stopspeed ? ph.stopspeed : speed;
      drop += fric * (control * frametime);
    }
    ns = speed - drop;
    if (ns < 0) ns = 0;
    ns /= speed;
    float nv[3];
    nv[0] = static_cast<float>(v[0] * ns);        // first component in double,
    nv[1] = v[1] * static_cast<float>(ns);        // the others in float
    nv[2] = v[2] * static_cast<float>(ns);
    copy3(v, nv);
  }
  SURF_HD void accelerate(const float* wishdir, double wishspeed, float accel) {
    if (st->waterjumptime) return;
    double cur = dot_d(st->velocity, wishdir);
    float add = static_cast<float>(wishspeed - cur);
    if (add <= 0) return;
    double acc = accel * frametime * wishspeed * pfriction;
    if (acc > add) acc = add;
    for (int i = 0; i < 3; ++i) st->velocity[i] = static_cast<float>(st->velocity[i] + acc * wishdir[i]);
  }
  // Air acceleration: the 30 u/s wish cap applies to the gain test only.
  SURF_HD void air_accelerate(const float* wishdir, float wishspeed, float accel) {
    if (st->waterjumptime) return;
    float capped = wishspeed > 30 ? 30 : wishspeed;
    double cur = dot_d(st->velocity, wishdir);
    float add = static_cast<float>(capped - cur);
    if (add <= 0) return;
    float acc_f = accel * wishspeed * frametime * pfriction;
    double acc = acc_f;
    if (acc > add) acc = add;
    for (int i = 0; i < 3; ++i) st->velocity[i] = static_cast<float>(st->velocity[i] + acc * wishdir[i]);
  }

  // FlyMove: up to four bumps, clipping velocity against the planes hit.
  SURF_HD int fly_move() {
    int blocked = 0, nplanes = 0;
    float planes[kMaxClipPlanes][3];
    float primal[3], original[3], nv[3], end[3], dir[3];
    Trace tr;
    float time_left = frametime, all_frac = 0;
    copy3(original, st->velocity);
    copy3(primal, st->velocity);
    for (int bump = 0; bump < 4; ++bump) {
      if (!st->velocity[0] && !st->velocity[1] && !st->velocity[2]) break;
      for (int i = 0; i < 3; ++i) {
        double step = time_left * st->velocity[i];
        end[i] = static_cast<float>(st->origin[i] + step);
      }
      trace(usehull, st->origin, end, &tr);
      all_frac += tr.fraction;
      if (tr.allsolid) {
        zero3(st->velocity);
        blocked_solid = true;
        return 4;
      }
      if (tr.fraction > 0.0f) {
        copy3(st->origin, tr.endpos);
        copy3(original, st->velocity);
        nplanes = 0;
      }
      if (tr.fraction == 1.0f) break;
      if (tr.normal[2] > 0.7f) blocked |= 1;
      if (!tr.normal[2]) blocked |= 2;
      time_left -= time_left * tr.fraction;
      if (nplanes >= kMaxClipPlanes) { zero3(st->velocity); break; }
      copy3(planes[nplanes], tr.normal);
      ++nplanes;
      if (nplanes == 1 && (st->onground == -1 || pfriction != 1)) {
        // airborne first impact: one clip (bounce only off non-floors)
        for (int i = 0; i < nplanes; ++i) {
          if (planes[i][2] > 0.7f) {
            clip_velocity(original, planes[i], nv, 1);
            copy3(original, nv);
          } else {
            clip_velocity(original, planes[i], nv, static_cast<float>(1.0 + ph.bounce * (1.0 - pfriction)));
          }
        }
        copy3(st->velocity, nv);
        copy3(original, nv);
      } else {
        int i, j;
        for (i = 0; i < nplanes; ++i) {
          clip_velocity(original, planes[i], st->velocity, 1);
          for (j = 0; j < nplanes; ++j)
            if (j != i && dot_d(st->velocity, planes[j]) < 0) break;
          if (j == nplanes) break;
        }
        if (i == nplanes) {
          if (nplanes != 2) { zero3(st->velocity); break; }
          // slide along the crease of the two planes (direction not normalized)
          dir[0] = planes[0][1] * planes[1][2] - planes[0][2] * planes[1][1];
          dir[1] = planes[0][2] * planes[1][0] - planes[0][0] * planes[1][2];
          dir[2] = planes[0][0] * planes[1][1] - planes[0][1] * planes[1][0];
          float d = static_cast<float>(dot_d(dir, st->velocity));
          st->velocity[0] = d * dir[0];
          st->velocity[1] = d * dir[1];
          st->velocity[2] = d * dir[2];
        }
        if (dot_d(st->velocity, primal) <= 0) { zero3(st->velocity); break; }
      }
    }
    if (all_frac == 0.0f) zero3(st->velocity);
    return blocked;
  }

  SURF_HD void wish_velocity(float* wishvel) {
    forward[2] = 0;
    right[2] = 0;
    normalize(forward);
    normalize(right);
    for (int i = 0; i < 2; ++i) wishvel[i] = forward[i] * fmove + right[i] * smove;
    wishvel[2] = 0;
  }

  // WalkMove: accelerate on the ground, then try the flat slide vs. a step-up.
  SURF_HD void walk_move() {
    float wishvel[3], wishdir[3], dest[3], orig[3], origvel[3], down[3], downvel[3], upp[3];
    Trace tr;
    if (ph.enable_stamina && st->fuser2 > 0.0) {
      double ratio = (100 - st->fuser2 * 0.001 * 19) * 0.01;
      st->velocity[0] = static_cast<float>(st->velocity[0] * ratio);
      st->velocity[1] = static_cast<float>(st->velocity[1] * ratio);
    }
    wish_velocity(wishvel);
    copy3(wishdir, wishvel);
    double wishspeed = normalize(wishdir);
    if (wishspeed > maxspeed) {
      float scale = static_cast<float>(maxspeed / wishspeed);
      for (int i = 0; i < 3; ++i) wishvel[i] *= scale;
      wishspeed = maxspeed;
    }
    st->velocity[2] = 0;
    accelerate(wishdir, wishspeed, ph.accelerate);
    st->velocity[2] = 0;
    for (int i = 0; i < 3; ++i) st->velocity[i] += st->basevelocity[i];
    double spd = length_d(st->velocity);
    if (spd < 1.0) { zero3(st->velocity); return; }
    int old_ground = st->onground;
    dest[0] = st->origin[0] + st->velocity[0] * frametime;
    dest[1] = st->origin[1] + st->velocity[1] * frametime;
    dest[2] = st->origin[2];
    trace(usehull, st->origin, dest, &tr);
    if (tr.fraction == 1.0f) { copy3(st->origin, tr.endpos); return; }
    if (old_ground == -1 && waterlevel == 0) return;
    copy3(orig, st->origin);
    copy3(origvel, st->velocity);
    fly_move();                                   // (a) slide at floor height
    copy3(down, st->origin);
    copy3(downvel, st->velocity);
    copy3(st->origin, orig);                      // (b) lift by stepsize, slide, press down
    copy3(st->velocity, origvel);
    copy3(dest, st->origin);
    dest[2] += ph.stepsize;
    trace(usehull, st->origin, dest, &tr);
    if (!tr.startsolid && !tr.allsolid) copy3(st->origin, tr.endpos);
    fly_move();
    copy3(dest, st->origin);
    dest[2] -= ph.stepsize;
    trace(usehull, st->origin, dest, &tr);
    bool use_down = tr.normal[2] < 0.7f;
    if (!use_down) {
      if (!tr.startsolid && !tr.allsolid) copy3(st->origin, tr.endpos);
      copy3(upp, st->origin);
      float dd = (down[0] - orig[0]) * (down[0] - orig[0]) + (down[1] - orig[1]) * (down[1] - orig[1]);
      float ud = (upp[0] - orig[0]) * (upp[0] - orig[0]) + (upp[1] - orig[1]) * (upp[1] - orig[1]);
      if (dd > ud) use_down = true;
      else st->velocity[2] = downvel[2];
    }
    if (use_down) {
      copy3(st->origin, down);
      copy3(st->velocity, downvel);
    }
  }

  SURF_HD void air_move() {
    float wishvel[3], wishdir[3];
    wish_velocity(wishvel);
    copy3(wishdir, wishvel);
    float wishspeed = static_cast<float>(normalize(wishdir));
    if (wishspeed > maxspeed) {
      float scale = maxspeed / wishspeed;
      for (int i = 0; i < 3; ++i) wishvel[i] *= scale;
      wishspeed = maxspeed;
    }
    air_accelerate(wishdir, wishspeed, ph.airaccelerate);
    for (int i = 0; i < 3; ++i) st->velocity[i] += st->basevelocity[i];
    fly_move();
  }

  SURF_HD static bool liquid(int c) { return contents_liquid(c); }

  // CheckWater: sample feet, body centre and eyes for liquid contents.
  SURF_HD void check_water() {
    float p[3];
    waterlevel = 0;
    watertype = kEmpty;
    if (!map.any_liquid) return;             // no probe could find a liquid (same result)
    p[0] = st->origin[0] + (player_mins(usehull, 0) + player_maxs(usehull, 0)) * 0.5f;
    p[1] = st->origin[1] + (player_mins(usehull, 1) + player_maxs(usehull, 1)) * 0.5f;
    p[2] = st->origin[2] + player_mins(usehull, 2) + 1;
    int c = point_contents(map, p);
    if (liquid(c)) {
      watertype = c;
      waterlevel = 1;
      float height = player_mins(usehull, 2) + player_maxs(usehull, 2);
      float half = height * 0.5f;
      p[2] = st->origin[2] + half;
      c = point_contents(map, p);
      if (liquid(c)) {
        waterlevel = 2;
        p[2] = st->origin[2] + view_ofs;
        c = point_contents(map, p);
        if (liquid(c)) waterlevel = 3;
      }
    }
  }

  // The down-trace of categorize(), through the player's GroundMemo if any.
  SURF_HD void ground_trace(const float* p, Trace* tr) {
    if (!ground) {
      trace(usehull, st->origin, p, tr);
      return;
    }
    uint32_t key[3];
    memcpy(key, st->origin, sizeof key);
    if (ground->hull == usehull && key[0] == ground->key[0] && key[1] == ground->key[1] && key[2] == ground->key[2]) {
      *tr = ground->tr;
      return;
    }
    trace(usehull, st->origin, p, tr);
    ground->hull = usehull;
    memcpy(ground->key, key, sizeof key);
    ground->tr = *tr;
  }

  // CategorizePosition: grounded iff a 2u down-trace hits a floor (n_z >= 0.7)
  // and we are not moving up faster than 180 u/s; snap onto it.
  SURF_HD void categorize() {
    float p[3];
    Trace tr;
    check_water();
    p[0] = st->origin[0];
    p[1] = st->origin[1];
    p[2] = st->origin[2] - 2;
    if (st->velocity[2] > 180) { st->onground = -1; return; }
    ground_trace(p, &tr);
    st->onground = tr.normal[2] < 0.7f ? -1 : tr.ent;
    if (st->onground != -1 && waterlevel < 2 && !tr.startsolid && !tr.allsolid) copy3(st->origin, tr.endpos);
  }

  // CheckStuck (server variant): one throttled nudge attempt per 5 ticks;
  // only the second half of the table may move the player.
  SURF_HD bool check_stuck() {
    if (position_free(st->origin)) { memo->index = 0; return false; }
    float base[3], test[3];
    copy3(base, st->origin);
    if (memo->last_tick != 0 && st->tick + 1 - memo->last_tick < 5) return true;
    memo->last_tick = st->tick + 1;
    int i = memo->index++ % 54;
    for (int k = 0; k < 3; ++k) test[k] = base[k] + stuck_offset(i, k);
    if (position_free(test)) {
      memo->index = 0;
      if (i >= 27) copy3(st->origin, test);
      return false;
    }
    return true;
  }

  SURF_HD void water_move() {
    float wishvel[3], wishdir[3], a[3], dest[3], tmp[3];
    Trace tr;
    double speed, accelspeed, wishspeed;
    float newspeed, addspeed;
    for (int i = 0; i < 3; ++i) wishvel[i] = forward[i] * fmove + smove * right[i];
    if (!fmove && !smove && !upmove) wishvel[2] -= 60.0f;     // sink when idle
    else wishvel[2] += upmove;
    copy3(wishdir, wishvel);
    wishspeed = normalize(wishdir);
    if (wishspeed > maxspeed) {
      float scale = static_cast<float>(maxspeed / wishspeed);
      for (int i = 0; i < 3; ++i) wishvel[i] *= scale;
      wishspeed = maxspeed;
    }
    wishspeed *= 0.8;
    for (int i = 0; i < 3; ++i) st->velocity[i] += st->basevelocity[i];
    copy3(tmp, st->velocity);
    speed = normalize(tmp);
    if (speed) {
      newspeed = static_cast<float>(speed - static_cast<double>(ph.friction * pfriction * frametime) * speed);
      if (newspeed < 0.0f) newspeed = 0.0f;
      float scale = static_cast<float>(newspeed / speed);
      for (int i = 0; i < 3; ++i) st->velocity[i] *= scale;
    } else {
      newspeed = 0;
    }
    if (static_cast<float>(wishspeed) < 0.1f) return;
    addspeed = static_cast<float>(static_cast<float>(wishspeed) - newspeed);
    if (addspeed > 0.0f) {
      normalize(wishvel);
      float acc_f = ph.accelerate * pfriction * frametime * static_cast<float>(wishspeed);
      accelspeed = acc_f;
      if (accelspeed > addspeed) accelspeed = addspeed;
      for (int i = 0; i < 3; ++i) st->velocity[i] = static_cast<float>(st->velocity[i] + accelspeed * wishvel[i]);
    }
    for (int i = 0; i < 3; ++i) dest[i] = st->origin[i] + frametime * st->velocity[i];
    copy3(a, dest);
    a[2] += ph.stepsize + 1;
    trace(usehull, a, dest, &tr);
    if (!tr.startsolid && !tr.allsolid) { copy3(st->origin, tr.endpos); return; }
    fly_move();
  }

  // CheckWaterJump: facing a near-vertical wall with clear space above it.
  SURF_HD void check_water_jump() {
    float a[3], b[3], flat_fwd[3], flat_vel[3];
    Trace tr;
    if (st->waterjumptime) return;
    if (st->velocity[2] < -180) return;
    flat_vel[0] = st->velocity[0];
    flat_vel[1] = st->velocity[1];
    flat_vel[2] = 0;
    double cur = normalize(flat_vel);
    flat_fwd[0] = forward[0];
    flat_fwd[1] = forward[1];
    flat_fwd[2] = 0;
    normalize(flat_fwd);
    if (cur != 0.0 && dot_d(flat_vel, flat_fwd) < 0.0) return;
    copy3(a, st->origin);
    a[2] += kWaterJumpHeight;
    for (int i = 0; i < 3; ++i) b[i] = a[i] + 24 * flat_fwd[i];
    int saved = usehull;
    usehull = 2;
    trace(2, a, b, &tr);
    if (tr.fraction < 1.0f && std::fabs(static_cast<double>(tr.normal[2])) < 0.1f) {
      a[2] += player_maxs(saved, 2) - kWaterJumpHeight;
      for (int i = 0; i < 3; ++i) {
        b[i] = a[i] + 24 * flat_fwd[i];
        st->movedir[i] = -50 * tr.normal[i];
      }
      trace(2, a, b, &tr);
      if (tr.fraction == 1.0f) {
        st->waterjumptime = 2000.0f;
        st->velocity[2] = 225.0f;
        st->oldbuttons |= kInJump;
      }
    }
    usehull = saved;
  }

  SURF_HD void water_jump() {
    if (st->waterjumptime > 10000) st->waterjumptime = 10000;
    if (!st->waterjumptime) return;
    st->waterjumptime -= msec;
    if (st->waterjumptime < 0 || !waterlevel) st->waterjumptime = 0;
    st->velocity[0] = st->movedir[0];
    st->velocity[1] = st->movedir[1];
  }

  // Ladder scan: first ladder volume whose hull (for the current usehull) contains us.
  SURF_HD int find_ladder() const {
    for (int i = 0; i < map.volumes.size(); ++i) {
      const BrushEntity& e = map.volumes[i];
      if (e.contents != kLadder) continue;
      if (st->origin[0] < e.absmin[0] - 20 || st->origin[0] > e.absmax[0] + 20 ||
          st->origin[1] < e.absmin[1] - 20 || st->origin[1] > e.absmax[1] + 20 ||
          st->origin[2] < e.absmin[2] - 40 || st->origin[2] > e.absmax[2] + 40)
        continue;
      HullView h = map.hull(e.model, bsp_hull_of_usehull(usehull));
      float local[3];
      for (int k = 0; k < 3; ++k) local[k] = st->origin[k] - (h.clip_mins[k] - player_mins(usehull, k) + e.origin[k]);
      if (hull_point_contents(h, h.first, local) != kEmpty) return i;
    }
    return -1;
  }

  SURF_HD void ladder_move(int idx, int* movetype) {
    const BrushEntity& lad = map.volumes[idx];
    const Model& mod = map.models[lad.model];
    float centre[3], floor_p[3];
    Trace tr;
    for (int i = 0; i < 3; ++i) centre[i] = (mod.mins[i] + mod.maxs[i]) * 0.5f;
    *movetype = kFly;
    copy3(floor_p, st->origin);
    floor_p[2] += player_mins(usehull, 2) - 1;
    bool on_floor = point_contents(map, floor_p) == kSolid;
    trace_model(map, lad.model, lad.origin, 2, st->origin, centre, &tr);
    if (tr.fraction == 1.0f) return;
    float fwd = 0, side = 0;
    float vpn[3], vr[3], vu[3];
    float climb = kMaxClimbSpeed;
    if (climb > maxspeed) climb = maxspeed;
    angle_vectors(angles, vpn, vr, vu);
    if (st->ducked) climb = static_cast<float>(climb * kDuckSpeedMult);
    if (buttons & kInBack) fwd -= climb;
    if (buttons & kInForward) fwd += climb;
    if (buttons & kInMoveLeft) side -= climb;
    if (buttons & kInMoveRight) side += climb;
    if (buttons & kInJump) {                          // let go: push off the face
      *movetype = kWalk;
      for (int i = 0; i < 3; ++i) st->velocity[i] = tr.normal[i] * 270;
    } else if (fwd != 0 || side != 0) {
      float vel[3], perp[3], into[3], lateral[3], tmp[3];
      const float* n = tr.normal;
      for (int i = 0; i < 3; ++i) vel[i] = vpn[i] * fwd + side * vr[i];
      zero3(tmp);
      tmp[2] = 1;
      perp[0] = tmp[1] * n[2] - tmp[2] * n[1];
      perp[1] = tmp[2] * n[0] - tmp[0] * n[2];
      perp[2] = tmp[0] * n[1] - tmp[1] * n[0];
      normalize(perp);
      float normal = static_cast<float>(dot_d(vel, n));
      for (int i = 0; i < 3; ++i) into[i] = n[i] * normal;
      for (int i = 0; i < 3; ++i) lateral[i] = vel[i] - into[i];
      tmp[0] = n[1] * perp[2] - n[2] * perp[1];
      tmp[1] = n[2] * perp[0] - n[0] * perp[2];
      tmp[2] = n[0] * perp[1] - n[1] * perp[0];
      for (int i = 0; i < 3; ++i) st->velocity[i] = lateral[i] + -normal * tmp[i];
      if (on_floor && normal > 0)
        for (int i = 0; i < 3; ++i) st->velocity[i] += kMaxClimbSpeed * n[i];
    } else {
      zero3(st->velocity);
    }
  }

  SURF_HD void fix_crouch_stuck(int direction) {
    float saved[3];
    if (position_free(st->origin)) return;
    copy3(saved, st->origin);
    for (int i = 0; i < kCrouchStuckSteps; ++i) {
      st->origin[2] += direction;
      if (position_free(st->origin)) return;
    }
    copy3(st->origin, saved);
  }

  SURF_HD void unduck() {
    float np[3];
    copy3(np, st->origin);
    if (st->onground != -1) np[2] = static_cast<float>(np[2] + 18.0);
    if (player_point_solid(map, usehull, np)) return;
    usehull = 0;
    if (player_point_solid(map, 0, np)) { usehull = 1; return; }   // no headroom: stay ducked
    st->ducked = 0;
    st->induck = 0;
    view_ofs = kViewStand;
    st->duck_time = 0;
    copy3(st->origin, np);
    categorize();
  }

  SURF_HD void duck() {
    int changed = st->oldbuttons ^ buttons;
    int pressed = changed & buttons;
    if (buttons & kInDuck) st->oldbuttons |= kInDuck;
    else st->oldbuttons &= ~kInDuck;
    if (!(buttons & kInDuck) && !st->induck && !st->ducked) return;
    double mult = kDuckSpeedMult;
    fmove = static_cast<float>(fmove * mult);
    smove = static_cast<float>(smove * mult);
    upmove = static_cast<float>(upmove * mult);
    if (buttons & kInDuck) {
      if ((pressed & kInDuck) && !st->ducked) {
        st->duck_time = 1000;
        st->induck = 1;
      }
      if (st->induck && ((st->duck_time / 1000.0) <= (1.0 - kTimeToDuck) || st->onground == -1)) {
        usehull = 1;
        view_ofs = kViewDuck;
        st->ducked = 1;
        st->induck = 0;
        if (st->onground != -1) {
          st->origin[2] = static_cast<float>(st->origin[2] - 18.0);
          fix_crouch_stuck(1);
          categorize();
        }
      }
    } else {
      unduck();
    }
  }

  // PreventMegaBunnyJumping: above 1.2x maxspeed, scale to 0.8 of that cap.
  SURF_HD void limit_bunnyhop() {
    float cap = kBhopFactor * maxspeed;
    if (cap <= 0.0f) return;
    double spd = length_d(st->velocity);
    if (spd <= cap) return;
    float f = static_cast<float>((cap / spd) * 0.8);
    for (int i = 0; i < 3; ++i) st->velocity[i] *= f;
  }

  SURF_HD void jump() {
    if (st->waterjumptime != 0.0f) {
      st->waterjumptime -= msec;
      if (st->waterjumptime < 0) st->waterjumptime = 0;
      return;
    }
    if (waterlevel >= 2) {                              // swim up
      st->onground = -1;
      st->velocity[2] = watertype == kWater ? 100 : watertype == kSlime ? 80 : 50;
      return;
    }
    if (st->onground == -1) { st->oldbuttons |= kInJump; return; }
    if (st->oldbuttons & kInJump) return;             // must release between jumps
    if (st->induck && st->ducked) return;
    st->onground = -1;
    if (ph.enable_bhop_cap) limit_bunnyhop();
    st->velocity[2] = static_cast<float>(std::sqrt(2.0 * 800.0f * 45.0f));
    if (ph.enable_stamina) {
      if (st->fuser2 > 0.0f) {
        double ratio = (100.0 - st->fuser2 * 0.001 * 19.0) * 0.01;
        st->velocity[2] = static_cast<float>(st->velocity[2] * ratio);
      }
      st->fuser2 = static_cast<float>(1315.789429);
    }
    fixup_gravity();
    st->oldbuttons |= kInJump;
  }
};

}  // namespace mv

SURF_HD inline MoveResult PlayerMove::tick(PlayerState* st, StuckMemo* memo, float yaw, float pitch, float fmove,
                                           float smove, int buttons, int msec, GroundMemo* ground) const {
  using namespace mv;
  Mover c{map_, ph_, st, memo};
  c.ground = ground;
  c.usehull = (ph_.enable_duck && st->ducked) ? 1 : 0;
  c.view_ofs = (ph_.enable_duck && st->ducked) ? kViewDuck : kViewStand;
  c.buttons = buttons;
  if (fmove > 0) c.buttons |= kInForward;             // clients set these from held keys
  else if (fmove < 0) c.buttons |= kInBack;
  if (smove > 0) c.buttons |= kInMoveRight;
  else if (smove < 0) c.buttons |= kInMoveLeft;
  c.msec = msec;
  c.fmove = fmove;
  c.smove = smove;
  c.upmove = 0;
  c.maxspeed = ph_.maxspeed;

  // CheckParameters: clamp the command to the effective max speed.
  float spd = static_cast<float>(std::sqrt(static_cast<double>(c.smove * c.smove + c.fmove * c.fmove + c.upmove * c.upmove)));
  double client_max = ph_.player_maxspeed;
  if (client_max != 0.0f) c.maxspeed = static_cast<float>(client_max < static_cast<double>(c.maxspeed) ? client_max : static_cast<double>(c.maxspeed));
  if (spd != 0.0f && spd > static_cast<double>(c.maxspeed)) {
    double ratio = static_cast<double>(c.maxspeed / spd);
    c.fmove = static_cast<float>(c.fmove * ratio);
    c.smove = static_cast<float>(c.smove * ratio);
    c.upmove = static_cast<float>(c.upmove * ratio);
  }
  c.angles[0] = pitch;
  c.angles[1] = yaw;
  c.angles[2] = 0;
  if (c.angles[1] > 180.0f) c.angles[1] -= 360.0f;

  // frame time and timers
  c.frametime = static_cast<float>(msec * 0.001);
  if (st->duck_time > 0) {
    st->duck_time -= msec;
    if (st->duck_time < 0) st->duck_time = 0;
  }
  if (st->fuser2 > 0.0) {
    st->fuser2 -= msec;
    if (st->fuser2 < 0.0) st->fuser2 = 0;
  }
  angle_vectors(c.angles, c.forward, c.right, c.up);

  MoveResult res;
  if (c.check_stuck()) {
    res.waterlevel = 0;
    res.blocked = true;
    return res;
  }
  c.categorize();
  int ladder = c.find_ladder();
  if (ph_.enable_duck) c.duck();
  int movetype = kWalk;
  if (ladder >= 0) c.ladder_move(ladder, &movetype);

  if (movetype == kFly) {
    c.check_water();
    if (!(c.buttons & kInJump)) st->oldbuttons &= ~kInJump;
    for (int i = 0; i < 3; ++i) st->velocity[i] += st->basevelocity[i];
    c.fly_move();
    for (int i = 0; i < 3; ++i) st->velocity[i] -= st->basevelocity[i];
  } else {
    if (!(c.waterlevel > 1)) c.add_gravity();
    if (st->waterjumptime != 0.0f) {
      c.water_jump();
      c.fly_move();
      c.check_water();
    } else if (c.waterlevel >= 2) {
      if (c.waterlevel == 2) c.check_water_jump();
      if (st->velocity[2] < 0 && st->waterjumptime) st->waterjumptime = 0;
      if (c.buttons & kInJump) c.jump();
      else st->oldbuttons &= ~kInJump;
      c.water_move();
      for (int i = 0; i < 3; ++i) st->velocity[i] -= st->basevelocity[i];
      c.categorize();
    } else {
      if (c.buttons & kInJump) c.jump();
      else st->oldbuttons &= ~kInJump;
      if (st->onground != -1) {
        st->velocity[2] = 0;
        c.friction();
      }
      c.check_velocity();
      if (st->onground != -1) c.walk_move();
      else c.air_move();
      c.categorize();
      for (int i = 0; i < 3; ++i) st->velocity[i] -= st->basevelocity[i];
      c.check_velocity();
      if (!(c.waterlevel > 1)) c.fixup_gravity();
      if (st->onground != -1) st->velocity[2] = 0;
    }
  }
  st->duck_time = static_cast<float>(static_cast<int>(st->duck_time));   // SV_RunCmd int writeback
  res.waterlevel = c.waterlevel;
  res.blocked = c.blocked_solid;
  return res;
}

}  // namespace surf
