// movement.hpp — Counter-Strike 1.6 player movement (pm_shared) over a Map.
//
// One call to PlayerMove::tick advances one player by one usercmd. The state
// layout is byte-compatible with the reference core's SurfState (108 bytes,
// src/surfcore.h:118-140) so state rows can be exchanged with it, recorded and
// restored. Precision discipline follows the published movement code: vec3
// storage is float, a handful of intermediate values are double ("real_t"),
// and every such site is marked where it happens.
#pragma once
#include <cstdint>

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

struct MoveResult { int waterlevel = 0; bool blocked = false; };

class PlayerMove {
 public:
  PlayerMove(const Map& map, const Physics& phys) : map_(map), ph_(phys) {}
  // yaw/pitch in GoldSrc convention (pitch + = down); fmove/smove in units.
  MoveResult tick(PlayerState* st, StuckMemo* memo, float yaw, float pitch, float fmove, float smove,
                  int buttons, int msec) const;

 private:
  const Map& map_;
  const Physics& ph_;
};

// The 54 nudge offsets of PM_CreateStuckTable, in engine order.
const float (*stuck_offsets())[3];

}  // namespace surf
