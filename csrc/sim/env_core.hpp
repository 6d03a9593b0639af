// env_core.hpp — the per-env rules of the vectorized surf env, header-only
// and SURF_HD: the host EnvBatch (C++ thread pool) and the GPU env (one CUDA
// thread per env) both run these functions over plain pointers, so a GPU
// rollout steps the same physics, triggers, rewards and resets.
//
// Behaviour matches the reference batch env (src/env.c:529-644): action
// decode, basevelocity fold, one pm tick, swept goal-box test, post-move
// triggers, fail rules, spline progress reward and same-step autoreset with a
// terminal observation.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

#include "movement.hpp"

namespace surf {

struct EnvConfig {                 // SurfEnvConfig-compatible (128 bytes)
  int32_t num_envs = 1;
  int32_t max_episode_ticks = 6000;
  int32_t lookahead_k = 8;
  float lookahead_dt = 0.25f;
  int32_t spawn_mode = 1;          // 0 map spawns, 1 spline curriculum, 2 spawn pool
  float spawn_curriculum_frac = 0.99f;
  float yaw_rate_max_deg = 10.f;
  float yaw_jitter_deg = 5.f;
  float kill_z = -1e38f;           // <= -1e30 -> world min z - 256
  int32_t water_fail = 1;
  float pitch_rate_max_deg = 10.f;
  int32_t lidar_w = 0, lidar_h = 0;
  float lidar_hfov_deg = 120.f, lidar_vfov_deg = 90.f, lidar_range = 2000.f;
  Physics phys;
  int32_t yaw_adaptive = 0;
};
static_assert(sizeof(EnvConfig) == 128, "EnvConfig layout");

constexpr int kObsFixed = 15;
constexpr int kActionDim = 6;
// Per-env record written by step_k (float32 columns).
enum RecCol : int {
  kRecOrigin = 0, kRecYaw = 3, kRecPitch = 4, kRecDucked = 5, kRecVel = 6, kRecTick = 9,
  kRecReward = 10, kRecDone = 11, kRecTrunc = 12, kRecGoal = 13, kRecEnded = 14, kRecOnground = 15,
  kRecCols = 16,
};
// Terminal pose of the last episode that ended inside a step_k call.
enum TermCol : int { kTermOrigin = 0, kTermYaw = 3, kTermPitch = 4, kTermDucked = 5, kTermTick = 6, kTermCols = 8 };

struct RowOut {                    // a strided float32 row target (nullptr = skip)
  float* ptr = nullptr;
  int64_t stride = 0;              // floats between consecutive env rows
  SURF_HD float* row(int i) const { return ptr + static_cast<int64_t>(i) * stride; }
};

namespace envk {

constexpr double kPiD = 3.14159265358979323846;

// Discrete view-turn ladders (degrees per tick at a 10 deg/tick rate limit),
// ascending so that the middle bin is "no turn". Action-space tables shared
// with the reference core (src/env.c:46-64) so policies are interchangeable.
SURF_HD inline float yaw_bin(int b) {
  const float t[15] = {-10.0f, -7.0f, -4.0f, -2.0f, -1.0f, -0.5f, -0.25f, 0.0f, 0.25f, 0.5f, 1.0f, 2.0f, 4.0f, 7.0f, 10.0f};
  return t[b];
}
// Adaptive yaw: multiples of the optimal-strafe turn rate atan(30/|v_h|).
SURF_HD inline float strafe_multiple(int b) {
  const float t[15] = {-20.0f, -8.0f, -3.0f, -1.5f, -1.0f, -0.75f, -0.5f, 0.0f, 0.5f, 0.75f, 1.0f, 1.5f, 3.0f, 8.0f, 20.0f};
  return t[b];
}
SURF_HD inline float pitch_bin(int b) {
  const float t[7] = {-10.0f, -5.0f, -2.0f, 0.0f, 2.0f, 5.0f, 10.0f};
  return t[b];
}

// SplitMix64 step and a 24-bit uniform in [0, 1).
SURF_HD inline uint64_t splitmix(uint64_t* s) {
  uint64_t z = (*s += 0x9E3779B97F4A7C15ULL);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
SURF_HD inline float uniform01(uint64_t* s) { return static_cast<float>((splitmix(s) >> 40) * (1.0 / 16777216.0)); }
SURF_HD inline float wrap360(float y) {
  y = std::fmod(y, 360.0f);
  if (y < 0) y += 360.0f;
  return y;
}
SURF_HD inline void copy3(float* d, const float* s) { d[0] = s[0]; d[1] = s[1]; d[2] = s[2]; }

// Swept segment vs AABB (slab test): thin finish curtains cannot be tunnelled.
SURF_HD inline bool segment_hits_box(const float* p0, const float* p1, const float* lo, const float* hi) {
  float t0 = 0.0f, t1 = 1.0f;
  for (int k = 0; k < 3; ++k) {
    float d = p1[k] - p0[k];
    if (d > -1e-9f && d < 1e-9f) {
      if (p0[k] < lo[k] || p0[k] > hi[k]) return false;
    } else {
      float a = (lo[k] - p0[k]) / d, b = (hi[k] - p0[k]) / d;
      if (a > b) { float t = a; a = b; b = t; }
      if (a > t0) t0 = a;
      if (b < t1) t1 = b;
      if (t0 > t1) return false;
    }
  }
  return true;
}

struct NoLidar {
  SURF_HD void operator()(const PlayerState&, float*) const {}
};

}  // namespace envk

// Everything one env step needs, as plain pointers (host vectors or device
// arrays). Per-env arrays are indexed by the env id.
struct EnvCore {
  EnvConfig cfg;
  MapView map;
  PlayerMove mover;
  float kill_z = 0, map_center[3] = {0, 0, 0};
  // progress spline (empty: no waypoints)
  Span<float> wp, cum, tang, tele_progress;
  float total_len = 0;
  Span<PlayerState> spawn_pool;
  int32_t teleport_fail = 0, goal_on = 0;
  float goal_min[3] = {0, 0, 0}, goal_max[3] = {0, 0, 0};
  // per-env state
  PlayerState* st = nullptr;
  StuckMemo* memo = nullptr;
  GroundMemo* ground = nullptr;    // host: per-env categorize cache (null on the GPU)
  float* last_yd = nullptr;
  float* last_pd = nullptr;
  uint64_t* rng = nullptr;
  uint64_t* push_used = nullptr;   // push_words per env: push-once trigger bitsets
  int32_t push_words = 1;
  uint8_t* goal_hit = nullptr;
  uint8_t* pending_fail = nullptr;

  struct TickOut { float reward; bool done, trunc, goal; };

  SURF_HD int nwp() const { return wp.size() / 3; }

  SURF_HD float yaw_delta(const PlayerState& s, int bin) const {
    if (!cfg.yaw_adaptive) return envk::yaw_bin(bin) * (cfg.yaw_rate_max_deg / 10.0f);
    float vh = std::sqrt(s.velocity[0] * s.velocity[0] + s.velocity[1] * s.velocity[1]);
    if (vh < 1.0f) vh = 1.0f;
    float w = std::atan(30.0f / vh) * (180.0f / 3.14159265358979f);
    float yd = envk::strafe_multiple(bin) * w;
    float lim = cfg.yaw_rate_max_deg;
    return yd > lim ? lim : (yd < -lim ? -lim : yd);
  }

  SURF_HD float spline_project(const float* p, int32_t* hint) const {
    int n = nwp();
    if (n < 2) return 0;
    int nseg = n - 1;
    if (*hint < 0) *hint = 0;
    if (*hint > nseg - 1) *hint = nseg - 1;
    int lo = *hint - 2, hi = *hint + 4;
    if (lo < 0) lo = 0;
    if (hi > nseg - 1) hi = nseg - 1;
    float best = 1e30f, prog = 0;
    int best_seg = *hint;
    for (int s = lo; s <= hi; ++s) {
      const float* a = &wp[3 * s];
      const float* b = &wp[3 * (s + 1)];
      float ab[3] = {b[0] - a[0], b[1] - a[1], b[2] - a[2]};
      float ap[3] = {p[0] - a[0], p[1] - a[1], p[2] - a[2]};
      float len2 = ab[0] * ab[0] + ab[1] * ab[1] + ab[2] * ab[2];
      float t = len2 > 0 ? (ap[0] * ab[0] + ap[1] * ab[1] + ap[2] * ab[2]) / len2 : 0;
      if (t < 0) t = 0; else if (t > 1) t = 1;
      float q[3] = {a[0] + ab[0] * t, a[1] + ab[1] * t, a[2] + ab[2] * t};
      float d[3] = {p[0] - q[0], p[1] - q[1], p[2] - q[2]};
      float d2 = d[0] * d[0] + d[1] * d[1] + d[2] * d[2];
      if (d2 < best) {
        best = d2;
        best_seg = s;
        prog = cum[s] + std::sqrt(len2) * t;
      }
    }
    *hint = best_seg;
    return prog;
  }

  SURF_HD void spline_sample(float u, float* pos, float* tg, int* seg_out) const {
    int n = nwp();
    if (u < 0) u = 0;
    if (u > total_len) u = total_len;
    int nseg = n - 1, s = 0;
    while (s < nseg - 1 && cum[s + 1] < u) ++s;
    float seglen = cum[s + 1] - cum[s];
    float t = seglen > 0 ? (u - cum[s]) / seglen : 0;
    const float* a = &wp[3 * s];
    const float* b = &wp[3 * (s + 1)];
    for (int i = 0; i < 3; ++i) pos[i] = a[i] + (b[i] - a[i]) * t;
    envk::copy3(tg, &tang[3 * s]);
    *seg_out = s;
  }

  SURF_HD void write_obs(const PlayerState& s, float lyd, float lpd, float* o) const {
    float yawr = s.yaw * static_cast<float>(envk::kPiD / 180.0);
    float cy = std::cos(yawr), sy = std::sin(yawr);
    float vx = s.velocity[0], vy = s.velocity[1], vz = s.velocity[2];
    o[0] = (vx * cy + vy * sy) / 1000.0f;          // ego frame: forward, left, up
    o[1] = (-vx * sy + vy * cy) / 1000.0f;
    o[2] = vz / 1000.0f;
    o[3] = std::sqrt(vx * vx + vy * vy) / 1000.0f;
    o[4] = s.onground != -1 ? 1.0f : 0.0f;
    o[5] = s.ducked ? 1.0f : 0.0f;
    o[6] = (s.oldbuttons & kInJump) ? 1.0f : 0.0f;
    o[7] = sy;
    o[8] = cy;
    o[9] = s.pitch / 90.0f;
    o[10] = cfg.yaw_rate_max_deg > 0 ? lyd / cfg.yaw_rate_max_deg : 0.0f;
    o[11] = cfg.pitch_rate_max_deg > 0 ? lpd / cfg.pitch_rate_max_deg : 0.0f;
    o[12] = (s.origin[0] - map_center[0]) / 2000.0f;
    o[13] = (s.origin[1] - map_center[1]) / 2000.0f;
    o[14] = (s.origin[2] - map_center[2]) / 2000.0f;
  }

  // ---- spawn / reset --------------------------------------------------------
  SURF_HD void reset_env(int i) const {
    PlayerState* s = &st[i];
    uint64_t* r = &rng[i];
    memset(s, 0, sizeof(*s));
    memo[i] = StuckMemo{};
    memset(&push_used[static_cast<int64_t>(i) * push_words], 0, sizeof(uint64_t) * static_cast<size_t>(push_words));
    last_yd[i] = 0;
    last_pd[i] = 0;
    s->onground = -1;
    const int n = nwp();
    if (cfg.spawn_mode == 2 && !spawn_pool.empty()) {
      int k = static_cast<int>(envk::splitmix(r) % static_cast<uint64_t>(spawn_pool.size()));
      *s = spawn_pool[k];
      s->tick = 0;
      s->stuck_ticks = 0;
      s->yaw = envk::wrap360(s->yaw + cfg.yaw_jitter_deg * (2.0f * envk::uniform01(r) - 1.0f));
      if (n >= 2) {
        if (s->seg_hint < 0 || s->seg_hint > n - 2) s->seg_hint = 0;
        s->progress = spline_project(s->origin, &s->seg_hint);
      } else {
        s->progress = 0;
      }
      s->best_progress = s->progress;
      return;
    }
    bool curriculum = cfg.spawn_mode == 1 && n >= 2 && envk::uniform01(r) < cfg.spawn_curriculum_frac;
    if (curriculum) {
      float u01 = envk::uniform01(r) * total_len * 0.98f;
      float pos[3], tg[3];
      int seg;
      spline_sample(u01, pos, tg, &seg);
      s->origin[0] = pos[0];
      s->origin[1] = pos[1];
      s->origin[2] = pos[2] + 20.0f;
      for (int k = 0; k < 3; ++k) s->velocity[k] = tg[k] * 250.0f;
      s->yaw = envk::wrap360(std::atan2(tg[1], tg[0]) * static_cast<float>(180.0 / envk::kPiD) +
                             cfg.yaw_jitter_deg * (2.0f * envk::uniform01(r) - 1.0f));
      s->seg_hint = seg;
      s->progress = s->best_progress = u01;
      float down[3] = {s->origin[0], s->origin[1], s->origin[2] - 40.0f};
      Trace tr;
      trace_player(map, 0, s->origin, down, &tr);
      if (tr.startsolid) s->origin[2] += 40.0f;
      else if (tr.fraction < 1.0f && tr.normal[2] >= 0.7f) envk::copy3(s->origin, tr.endpos);
    } else {
      int ns = map.spawns.empty() ? 1 : map.spawns.size();
      int k = static_cast<int>(envk::splitmix(r) % static_cast<uint64_t>(ns));
      if (!map.spawns.empty()) {
        envk::copy3(s->origin, map.spawns[k].origin);
        s->yaw = envk::wrap360(map.spawns[k].yaw + cfg.yaw_jitter_deg * (2.0f * envk::uniform01(r) - 1.0f));
      }
      s->seg_hint = 0;
      s->progress = s->best_progress = spline_project(s->origin, &s->seg_hint);
    }
  }

  // ---- triggers: 0 none, 1 fail, 2 benign teleport ---------------------------
  SURF_HD int apply_triggers(int env, PlayerState* s) const {
    const int uh = (cfg.phys.enable_duck && s->ducked) ? 1 : 0;
    const int n = nwp();
    for (int i = 0; i < map.triggers.size(); ++i) {
      const Trigger& t = map.triggers[i];
      if (s->origin[0] + player_maxs(uh, 0) < t.absmin[0] || s->origin[0] + player_mins(uh, 0) > t.absmax[0] ||
          s->origin[1] + player_maxs(uh, 1) < t.absmin[1] || s->origin[1] + player_mins(uh, 1) > t.absmax[1] ||
          s->origin[2] + player_maxs(uh, 2) < t.absmin[2] || s->origin[2] + player_mins(uh, 2) > t.absmax[2])
        continue;
      if (!trigger_contains(map, t, uh, s->origin)) continue;
      if (t.kind == TriggerKind::kHurt) {
        if (t.damage >= 90.0f) return 1;
      } else if (t.kind == TriggerKind::kPush) {
        if (t.push_once) {
          uint64_t* used = &push_used[static_cast<int64_t>(env) * push_words + (i >> 6)];
          uint64_t bit = 1ULL << (i & 63);
          if (!(*used & bit)) {
            *used |= bit;
            for (int k = 0; k < 3; ++k) s->velocity[k] += t.push_velocity[k];
            if (t.push_velocity[2] > 0) s->onground = -1;
          }
        } else {
          float push[3];
          envk::copy3(push, t.push_velocity);
          if (s->base_vel_flag)
            for (int k = 0; k < 3; ++k) push[k] += s->basevelocity[k];
          envk::copy3(s->basevelocity, push);
          s->base_vel_flag = 1;
        }
      } else {                                           // teleport
        if (!t.has_dest) continue;                       // unresolved target: inert
        const float dest_prog = n >= 2 ? tele_progress[i] : 0.f;
        if (n >= 2 && dest_prog < s->progress - 500.0f) return 1;
        s->origin[0] = t.dest[0];
        s->origin[1] = t.dest[1];
        s->origin[2] = t.dest[2] - player_mins(uh, 2);
        s->origin[2] += 1.0f;
        s->yaw = envk::wrap360(t.dest_yaw);
        for (int k = 0; k < 3; ++k) s->velocity[k] = s->basevelocity[k] = 0;
        s->base_vel_flag = 0;
        s->onground = -1;
        if (n >= 2) {
          int nseg = n - 1, seg = 0;
          while (seg < nseg - 1 && cum[seg + 1] < dest_prog) ++seg;
          s->seg_hint = seg;
          s->progress = dest_prog;
        }
        return 2;
      }
    }
    return 0;
  }

  // ---- one tick of one env ----------------------------------------------------
  template <class Lidar>
  SURF_HD TickOut tick_env(int i, float yd, float pd, float fmove, float smove, int buttons, bool forced,
                           float* obs_row, float* term_row, float* term_rec, const Lidar& lidar) const {
    PlayerState* s = &st[i];
    s->yaw = envk::wrap360(s->yaw + yd);
    last_yd[i] = yd;
    s->pitch += pd;
    if (s->pitch > 30.0f) s->pitch = 30.0f;         // asymmetric view clamp
    if (s->pitch < -70.0f) s->pitch = -70.0f;
    last_pd[i] = pd;
    if (!s->base_vel_flag) {                        // moving-ground basevelocity fold
      float sc = static_cast<float>(cfg.phys.msec * 0.001) * 0.5f + 1.0f;
      for (int k = 0; k < 3; ++k) s->velocity[k] += sc * s->basevelocity[k];
      s->basevelocity[0] = s->basevelocity[1] = s->basevelocity[2] = 0.0f;
    }
    s->base_vel_flag = 0;
    goal_hit[i] = 0;
    forced = forced || pending_fail[i];
    pending_fail[i] = 0;
    float prev_org[3];
    envk::copy3(prev_org, s->origin);
    float prev_prog = s->progress;
    // View pitch never enters the movement tick (it aims the sensor only).
#if defined(__CUDA_ARCH__)
    GroundMemo* gm = nullptr;                          // host-only cache
#else
    GroundMemo* gm = ground ? &ground[i] : nullptr;
#endif
    MoveResult mr = mover.tick(s, &memo[i], s->yaw, 0.0f, fmove, smove, buttons, cfg.phys.msec, gm);
    s->tick++;
    bool fail = false, complete = false;
    if (goal_on) {
      const int uh = (cfg.phys.enable_duck && s->ducked) ? 1 : 0;
      float lo[3], hi[3];
      for (int k = 0; k < 3; ++k) { lo[k] = goal_min[k] - player_maxs(uh, k); hi[k] = goal_max[k] - player_mins(uh, k); }
      if (envk::segment_hits_box(prev_org, s->origin, lo, hi)) { complete = true; goal_hit[i] = 1; }
    }
    int trig = complete ? 0 : apply_triggers(i, s);
    if (trig == 1) fail = true;
    if (trig == 2 && teleport_fail) fail = true;
    if (forced && !complete) fail = true;
    float r = 0;
    const int n = nwp();
    if (n >= 2) {
      s->progress = spline_project(s->origin, &s->seg_hint);
      if (trig != 2) r = 0.05f * (s->progress - prev_prog);
      if (s->progress > s->best_progress) s->best_progress = s->progress;
      if (s->progress >= total_len - 50.0f) {
        const float* fin = &wp[3 * (n - 1)];
        float dx = s->origin[0] - fin[0], dy = s->origin[1] - fin[1], dz = s->origin[2] - fin[2];
        if (dx * dx + dy * dy + dz * dz < 150.0f * 150.0f) { complete = true; r += 50.0f; }
      }
    }
    if (mr.waterlevel >= 2 && cfg.water_fail) fail = true;
    if (s->origin[2] < kill_z) fail = true;
    s->stuck_ticks = mr.blocked ? s->stuck_ticks + 1 : 0;
    if (s->stuck_ticks >= 5) fail = true;
    bool truncated = s->tick >= cfg.max_episode_ticks;
    bool d = fail || complete;
    TickOut out{r, d, truncated && !d, complete};
    if (d || truncated) {
      if (term_row) {
        write_obs(*s, last_yd[i], last_pd[i], term_row);
        lidar(*s, term_row + kObsFixed);
      }
      if (term_rec) {
        envk::copy3(term_rec + kTermOrigin, s->origin);
        term_rec[kTermYaw] = s->yaw;
        term_rec[kTermPitch] = s->pitch;
        term_rec[kTermDucked] = static_cast<float>(s->ducked);
        term_rec[kTermTick] = static_cast<float>(s->tick);
      }
      reset_env(i);
      if (obs_row) {
        write_obs(st[i], 0.0f, 0.0f, obs_row);
        lidar(st[i], obs_row + kObsFixed);
      }
    } else if (obs_row) {
      write_obs(*s, last_yd[i], last_pd[i], obs_row);
      lidar(*s, obs_row + kObsFixed);
    }
    return out;
  }

  // K ticks of action repeat for env i (one row of step_k): decode the action
  // row, tick, reduce the per-tick signals and write the env's record row.
  template <class Lidar>
  SURF_HD void step_k_one(int i, const int32_t* a, int yaw_slot, int fail_slot, int k, RowOut obs, RowOut term_obs,
                          RowOut rec, RowOut term_rec, const Lidar& lidar) const {
    int pb = a[1] < 0 ? 0 : (a[1] > 6 ? 6 : a[1]);
    float pd = envk::pitch_bin(pb) * (cfg.pitch_rate_max_deg / 10.0f);
    float fm = a[2] <= 0 ? -400.0f : (a[2] >= 2 ? 400.0f : 0.0f);
    float sm = a[3] <= 0 ? -400.0f : (a[3] >= 2 ? 400.0f : 0.0f);
    int buttons = (a[4] ? kInJump : 0) | (a[5] ? kInDuck : 0);
    int yb = a[0] < 0 ? 0 : (a[0] > 14 ? 14 : a[0]);
    float yc = 0.f;
    if (yaw_slot >= 0) {
      memcpy(&yc, &a[yaw_slot], sizeof yc);
      yc = yc > 1.f ? 1.f : (yc < -1.f ? -1.f : yc);
      if (yc != yc) yc = 0.f;
    }
    bool forced = fail_slot >= 0 && a[fail_slot] != 0;
    float rsum = 0;
    bool done = false, trunc = false, goal = false;
    for (int j = 0; j < k; ++j) {
      float yd = yaw_slot >= 0 ? yc * cfg.yaw_rate_max_deg : yaw_delta(st[i], yb);
      float* orow = (j == k - 1 && obs.ptr) ? obs.row(i) : nullptr;
      TickOut t = tick_env(i, yd, pd, fm, sm, buttons, forced && j == 0, orow,
                           term_obs.ptr ? term_obs.row(i) : nullptr, term_rec.ptr ? term_rec.row(i) : nullptr, lidar);
      rsum += t.reward;
      done |= t.done;
      trunc |= t.trunc;
      goal |= t.goal;
    }
    if (rec.ptr) {
      const PlayerState& s = st[i];
      float* o = rec.row(i);
      envk::copy3(o + kRecOrigin, s.origin);
      o[kRecYaw] = s.yaw;
      o[kRecPitch] = s.pitch;
      o[kRecDucked] = static_cast<float>(s.ducked);
      envk::copy3(o + kRecVel, s.velocity);
      o[kRecTick] = static_cast<float>(s.tick);
      o[kRecReward] = rsum;
      o[kRecDone] = done ? 1.f : 0.f;
      o[kRecTrunc] = trunc ? 1.f : 0.f;
      o[kRecGoal] = goal ? 1.f : 0.f;
      o[kRecEnded] = (done || trunc) ? 1.f : 0.f;
      o[kRecOnground] = s.onground != -1 ? 1.f : 0.f;
    }
  }

  // Seed env i's stream and spawn it (reset_all's per-env body).
  SURF_HD void seed_and_reset(int i, uint64_t seed) const {
    uint64_t t = seed + static_cast<uint64_t>(i);      // per-env stream through the mixer
    rng[i] = envk::splitmix(&t) | 1;
    reset_env(i);
  }
};

}  // namespace surf
