// env.cpp — vectorized env. See env.hpp.
#include "env.hpp"

#include <cmath>
#include <cstring>

namespace surf {
namespace {

constexpr double kPiD = 3.14159265358979323846;
// Discrete view-turn ladders (degrees per tick at a 10 deg/tick rate limit),
// ascending so that the middle bin is "no turn". Action-space tables shared
// with the reference core (src/env.c:46-64) so policies are interchangeable.
constexpr float kYawBins[15] = {-10.0f, -7.0f, -4.0f, -2.0f, -1.0f, -0.5f, -0.25f, 0.0f,
                                0.25f, 0.5f, 1.0f, 2.0f, 4.0f, 7.0f, 10.0f};
// Adaptive yaw: multiples of the optimal-strafe turn rate atan(30/|v_h|).
constexpr float kStrafeMultiples[15] = {-20.0f, -8.0f, -3.0f, -1.5f, -1.0f, -0.75f, -0.5f, 0.0f,
                                        0.5f, 0.75f, 1.0f, 1.5f, 3.0f, 8.0f, 20.0f};
constexpr float kPitchBins[7] = {-10.0f, -5.0f, -2.0f, 0.0f, 2.0f, 5.0f, 10.0f};

// SplitMix64 step and a 24-bit uniform in [0, 1).
inline uint64_t splitmix(uint64_t* s) {
  uint64_t z = (*s += 0x9E3779B97F4A7C15ULL);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
inline float uniform01(uint64_t* s) { return static_cast<float>((splitmix(s) >> 40) * (1.0 / 16777216.0)); }
inline float wrap360(float y) {
  y = std::fmod(y, 360.0f);
  if (y < 0) y += 360.0f;
  return y;
}
inline void copy3(float* d, const float* s) { d[0] = s[0]; d[1] = s[1]; d[2] = s[2]; }

// Swept segment vs AABB (slab test): thin finish curtains cannot be tunnelled.
bool segment_hits_box(const float* p0, const float* p1, const float* lo, const float* hi) {
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

}  // namespace

EnvBatch::EnvBatch(std::shared_ptr<const Map> map, const EnvConfig& cfg, int threads)
    : map_(std::move(map)), cfg_(cfg), mover_(*map_, cfg_.phys) {
  if (cfg_.num_envs < 1) cfg_.num_envs = 1;
  if (cfg_.lookahead_k < 0) cfg_.lookahead_k = 0;
  if (cfg_.phys.msec < 1) cfg_.phys.msec = 1;
  if (cfg_.phys.msec > 50) cfg_.phys.msec = 50;
  if (cfg_.lidar_w < 0) cfg_.lidar_w = 0;
  if (cfg_.lidar_h < 0) cfg_.lidar_h = 0;
  if (cfg_.lidar_w == 0 || cfg_.lidar_h == 0) cfg_.lidar_w = cfg_.lidar_h = 0;
  if (cfg_.lidar_range <= 1.0f) cfg_.lidar_range = 2000.0f;
  if (cfg_.pitch_rate_max_deg < 0.0f) cfg_.pitch_rate_max_deg = 10.0f;
  obs_dim_ = kObsFixed + cfg_.lidar_w * cfg_.lidar_h;
  kill_z_ = cfg_.kill_z <= -1e30f ? map_->world_mins[2] - 256.0f : cfg_.kill_z;
  for (int k = 0; k < 3; ++k) map_center_[k] = 0.5f * (map_->world_mins[k] + map_->world_maxs[k]);
  const size_t n = static_cast<size_t>(cfg_.num_envs);
  st_.assign(n, PlayerState{});
  memo_.assign(n, StuckMemo{});
  last_yd_.assign(n, 0.f);
  last_pd_.assign(n, 0.f);
  rng_.assign(n, 0);
  push_words_ = static_cast<int>((map_->triggers.size() + 63) / 64);
  if (push_words_ < 1) push_words_ = 1;
  push_used_.assign(n * static_cast<size_t>(push_words_), 0);
  goal_hit_.assign(n, 0);
  pending_fail_.assign(n, 0);
  pool_ = std::make_unique<ThreadPool>(threads);
}

float EnvBatch::yaw_delta(const PlayerState& s, int bin) const {
  if (!cfg_.yaw_adaptive) return kYawBins[bin] * (cfg_.yaw_rate_max_deg / 10.0f);
  float vh = std::sqrt(s.velocity[0] * s.velocity[0] + s.velocity[1] * s.velocity[1]);
  if (vh < 1.0f) vh = 1.0f;
  float w = std::atan(30.0f / vh) * (180.0f / 3.14159265358979f);
  float yd = kStrafeMultiples[bin] * w;
  float lim = cfg_.yaw_rate_max_deg;
  return yd > lim ? lim : (yd < -lim ? -lim : yd);
}

// ---- progress spline -------------------------------------------------------
float EnvBatch::spline_project(const float* p, int32_t* hint) const {
  int nwp = static_cast<int>(wp_.size() / 3);
  if (nwp < 2) return 0;
  int nseg = nwp - 1;
  if (*hint < 0) *hint = 0;
  if (*hint > nseg - 1) *hint = nseg - 1;
  int lo = *hint - 2, hi = *hint + 4;
  if (lo < 0) lo = 0;
  if (hi > nseg - 1) hi = nseg - 1;
  float best = 1e30f, prog = 0;
  int best_seg = *hint;
  for (int s = lo; s <= hi; ++s) {
    const float* a = &wp_[3 * s];
    const float* b = &wp_[3 * (s + 1)];
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
      prog = cum_[s] + std::sqrt(len2) * t;
    }
  }
  *hint = best_seg;
  return prog;
}

void EnvBatch::spline_sample(float u, float* pos, float* tang, int* seg_out) const {
  int nwp = static_cast<int>(wp_.size() / 3);
  if (u < 0) u = 0;
  if (u > total_len_) u = total_len_;
  int nseg = nwp - 1, s = 0;
  while (s < nseg - 1 && cum_[s + 1] < u) ++s;
  float seglen = cum_[s + 1] - cum_[s];
  float t = seglen > 0 ? (u - cum_[s]) / seglen : 0;
  const float* a = &wp_[3 * s];
  const float* b = &wp_[3 * (s + 1)];
  for (int i = 0; i < 3; ++i) pos[i] = a[i] + (b[i] - a[i]) * t;
  copy3(tang, &tang_[3 * s]);
  *seg_out = s;
}

int EnvBatch::set_waypoints(const float* xyz, int count) {
  if (!xyz || count < 2) return -1;
  wp_.assign(xyz, xyz + 3 * count);
  cum_.assign(static_cast<size_t>(count), 0.f);
  tang_.assign(static_cast<size_t>(3 * count), 0.f);
  for (int i = 0; i < count - 1; ++i) {
    float d[3] = {wp_[3 * (i + 1)] - wp_[3 * i], wp_[3 * (i + 1) + 1] - wp_[3 * i + 1], wp_[3 * (i + 1) + 2] - wp_[3 * i + 2]};
    float len = std::sqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
    if (len < 1e-3f) len = 1e-3f;
    for (int k = 0; k < 3; ++k) tang_[3 * i + k] = d[k] / len;
    cum_[i + 1] = cum_[i] + len;
  }
  copy3(&tang_[3 * (count - 1)], &tang_[3 * (count - 2)]);
  total_len_ = cum_[count - 1];
  // Teleport destination progress: global projection over every segment.
  tele_progress_.assign(map_->triggers.size(), 0.f);
  for (size_t ti = 0; ti < map_->triggers.size(); ++ti) {
    const Trigger& t = map_->triggers[ti];
    if (t.kind != TriggerKind::kTeleport || !t.has_dest) continue;
    float best = 1e30f, prog = 0;
    for (int s = 0; s < count - 1; ++s) {
      const float* a = &wp_[3 * s];
      const float* b = &wp_[3 * (s + 1)];
      float ab[3] = {b[0] - a[0], b[1] - a[1], b[2] - a[2]};
      float ap[3] = {t.dest[0] - a[0], t.dest[1] - a[1], t.dest[2] - a[2]};
      float len2 = ab[0] * ab[0] + ab[1] * ab[1] + ab[2] * ab[2];
      float tt = len2 > 0 ? (ap[0] * ab[0] + ap[1] * ab[1] + ap[2] * ab[2]) / len2 : 0;
      if (tt < 0) tt = 0; else if (tt > 1) tt = 1;
      float q[3] = {a[0] + ab[0] * tt, a[1] + ab[1] * tt, a[2] + ab[2] * tt};
      float dx = t.dest[0] - q[0], dy = t.dest[1] - q[1], dz = t.dest[2] - q[2];
      float d2 = dx * dx + dy * dy + dz * dz;
      if (d2 < best) { best = d2; prog = cum_[s] + std::sqrt(len2) * tt; }
    }
    tele_progress_[ti] = prog;
  }
  for (PlayerState& s : st_) {
    if (s.seg_hint < 0) s.seg_hint = 0;
    if (s.seg_hint > count - 2) s.seg_hint = count - 2;
    s.progress = spline_project(s.origin, &s.seg_hint);
    if (s.best_progress > total_len_) s.best_progress = s.progress;
  }
  return 0;
}

int EnvBatch::set_spawn_pool(const PlayerState* pool, int n) {
  if (!pool || n < 1) return -1;
  spawn_pool_.assign(pool, pool + n);
  return 0;
}

void EnvBatch::set_goal_box(const float* mins, const float* maxs) {
  if (!mins || !maxs) { goal_on_ = false; return; }
  copy3(goal_min_, mins);
  copy3(goal_max_, maxs);
  goal_on_ = true;
}

void EnvBatch::force_fail(const uint8_t* mask) {
  if (!mask) return;
  for (int i = 0; i < cfg_.num_envs; ++i)
    if (mask[i]) pending_fail_[static_cast<size_t>(i)] = 1;
}

void EnvBatch::set_state(int env, const PlayerState& s) {
  if (env < 0 || env >= cfg_.num_envs) return;
  st_[static_cast<size_t>(env)] = s;
  PlayerState& d = st_[static_cast<size_t>(env)];
  if (d.seg_hint < 0) d.seg_hint = 0;
  int nwp = static_cast<int>(wp_.size() / 3);
  if (nwp >= 2 && d.seg_hint > nwp - 2) d.seg_hint = nwp - 2;
}

// ---- observation -------------------------------------------------------------
void EnvBatch::write_lidar(const PlayerState& s, float* o) const {
  const int W = cfg_.lidar_w, H = cfg_.lidar_h;
  if (W <= 0 || H <= 0) return;
  float eye[3] = {s.origin[0], s.origin[1], s.origin[2] + (s.ducked ? 12.0f : 17.0f)};
  const float d2r = static_cast<float>(kPiD / 180.0);
  const float range = cfg_.lidar_range;
  for (int r = 0; r < H; ++r) {
    float poff = cfg_.lidar_vfov_deg * (0.5f - (r + 0.5f) / static_cast<float>(H));
    float p = (s.pitch + poff) * d2r;
    float cp = std::cos(p), sp = std::sin(p);
    for (int c = 0; c < W; ++c) {
      float yoff = cfg_.lidar_hfov_deg * (0.5f - (c + 0.5f) / static_cast<float>(W));
      float yw = (s.yaw + yoff) * d2r;
      float end[3] = {eye[0] + cp * std::cos(yw) * range, eye[1] + cp * std::sin(yw) * range, eye[2] + sp * range};
      Trace tr;
      trace_player(*map_, 2, eye, end, &tr);
      o[r * W + c] = tr.startsolid ? 0.0f : tr.fraction;
    }
  }
}

void EnvBatch::write_obs(const PlayerState& s, float last_yd, float last_pd, float* o) const {
  float yawr = s.yaw * static_cast<float>(kPiD / 180.0);
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
  o[10] = cfg_.yaw_rate_max_deg > 0 ? last_yd / cfg_.yaw_rate_max_deg : 0.0f;
  o[11] = cfg_.pitch_rate_max_deg > 0 ? last_pd / cfg_.pitch_rate_max_deg : 0.0f;
  o[12] = (s.origin[0] - map_center_[0]) / 2000.0f;
  o[13] = (s.origin[1] - map_center_[1]) / 2000.0f;
  o[14] = (s.origin[2] - map_center_[2]) / 2000.0f;
  write_lidar(s, o + kObsFixed);
}

// ---- spawn / reset --------------------------------------------------------
void EnvBatch::reset_env(int i) {
  const size_t u = static_cast<size_t>(i);
  PlayerState* s = &st_[u];
  uint64_t* r = &rng_[u];
  std::memset(s, 0, sizeof(*s));
  memo_[u] = StuckMemo{};
  std::memset(&push_used_[u * static_cast<size_t>(push_words_)], 0, sizeof(uint64_t) * static_cast<size_t>(push_words_));
  last_yd_[u] = 0;
  last_pd_[u] = 0;
  s->onground = -1;
  const int nwp = static_cast<int>(wp_.size() / 3);
  if (cfg_.spawn_mode == 2 && !spawn_pool_.empty()) {
    int k = static_cast<int>(splitmix(r) % static_cast<uint64_t>(spawn_pool_.size()));
    *s = spawn_pool_[static_cast<size_t>(k)];
    s->tick = 0;
    s->stuck_ticks = 0;
    s->yaw = wrap360(s->yaw + cfg_.yaw_jitter_deg * (2.0f * uniform01(r) - 1.0f));
    if (nwp >= 2) {
      if (s->seg_hint < 0 || s->seg_hint > nwp - 2) s->seg_hint = 0;
      s->progress = spline_project(s->origin, &s->seg_hint);
    } else {
      s->progress = 0;
    }
    s->best_progress = s->progress;
    return;
  }
  bool curriculum = cfg_.spawn_mode == 1 && nwp >= 2 && uniform01(r) < cfg_.spawn_curriculum_frac;
  if (curriculum) {
    float u01 = uniform01(r) * total_len_ * 0.98f;
    float pos[3], tg[3];
    int seg;
    spline_sample(u01, pos, tg, &seg);
    s->origin[0] = pos[0];
    s->origin[1] = pos[1];
    s->origin[2] = pos[2] + 20.0f;
    for (int k = 0; k < 3; ++k) s->velocity[k] = tg[k] * 250.0f;
    s->yaw = wrap360(std::atan2(tg[1], tg[0]) * static_cast<float>(180.0 / kPiD) +
                     cfg_.yaw_jitter_deg * (2.0f * uniform01(r) - 1.0f));
    s->seg_hint = seg;
    s->progress = s->best_progress = u01;
    float down[3] = {s->origin[0], s->origin[1], s->origin[2] - 40.0f};
    Trace tr;
    trace_player(*map_, 0, s->origin, down, &tr);
    if (tr.startsolid) s->origin[2] += 40.0f;
    else if (tr.fraction < 1.0f && tr.normal[2] >= 0.7f) copy3(s->origin, tr.endpos);
  } else {
    int ns = map_->spawns.empty() ? 1 : static_cast<int>(map_->spawns.size());
    int k = static_cast<int>(splitmix(r) % static_cast<uint64_t>(ns));
    if (!map_->spawns.empty()) {
      copy3(s->origin, map_->spawns[static_cast<size_t>(k)].origin);
      s->yaw = wrap360(map_->spawns[static_cast<size_t>(k)].yaw + cfg_.yaw_jitter_deg * (2.0f * uniform01(r) - 1.0f));
    }
    s->seg_hint = 0;
    s->progress = s->best_progress = spline_project(s->origin, &s->seg_hint);
  }
}

// ---- triggers: 0 none, 1 fail, 2 benign teleport ---------------------------
int EnvBatch::apply_triggers(int env, PlayerState* s) {
  const Map& m = *map_;
  const int uh = (cfg_.phys.enable_duck && s->ducked) ? 1 : 0;
  const int nwp = static_cast<int>(wp_.size() / 3);
  for (size_t i = 0; i < m.triggers.size(); ++i) {
    const Trigger& t = m.triggers[i];
    if (s->origin[0] + kPlayerMaxs[uh][0] < t.absmin[0] || s->origin[0] + kPlayerMins[uh][0] > t.absmax[0] ||
        s->origin[1] + kPlayerMaxs[uh][1] < t.absmin[1] || s->origin[1] + kPlayerMins[uh][1] > t.absmax[1] ||
        s->origin[2] + kPlayerMaxs[uh][2] < t.absmin[2] || s->origin[2] + kPlayerMins[uh][2] > t.absmax[2])
      continue;
    if (!trigger_contains(m, t, uh, s->origin)) continue;
    if (t.kind == TriggerKind::kHurt) {
      if (t.damage >= 90.0f) return 1;
    } else if (t.kind == TriggerKind::kPush) {
      if (t.push_once) {
        uint64_t* used = &push_used_[static_cast<size_t>(env) * static_cast<size_t>(push_words_) + (i >> 6)];
        uint64_t bit = 1ULL << (i & 63);
        if (!(*used & bit)) {
          *used |= bit;
          for (int k = 0; k < 3; ++k) s->velocity[k] += t.push_velocity[k];
          if (t.push_velocity[2] > 0) s->onground = -1;
        }
      } else {
        float push[3];
        copy3(push, t.push_velocity);
        if (s->base_vel_flag)
          for (int k = 0; k < 3; ++k) push[k] += s->basevelocity[k];
        copy3(s->basevelocity, push);
        s->base_vel_flag = 1;
      }
    } else {                                           // teleport
      if (!t.has_dest) continue;                       // unresolved target: inert
      const float dest_prog = nwp >= 2 ? tele_progress_[i] : 0.f;
      if (nwp >= 2 && dest_prog < s->progress - 500.0f) return 1;
      s->origin[0] = t.dest[0];
      s->origin[1] = t.dest[1];
      s->origin[2] = t.dest[2] - kPlayerMins[uh][2];
      s->origin[2] += 1.0f;
      s->yaw = wrap360(t.dest_yaw);
      for (int k = 0; k < 3; ++k) s->velocity[k] = s->basevelocity[k] = 0;
      s->base_vel_flag = 0;
      s->onground = -1;
      if (nwp >= 2) {
        int nseg = nwp - 1, seg = 0;
        while (seg < nseg - 1 && cum_[seg + 1] < dest_prog) ++seg;
        s->seg_hint = seg;
        s->progress = dest_prog;
      }
      return 2;
    }
  }
  return 0;
}

// ---- one tick of one env ----------------------------------------------------
EnvBatch::TickOut EnvBatch::tick_env(int i, float yd, float pd, float fmove, float smove, int buttons, bool forced,
                                     float* obs_row, float* term_row, float* term_rec) {
  const size_t u = static_cast<size_t>(i);
  PlayerState* s = &st_[u];
  s->yaw = wrap360(s->yaw + yd);
  last_yd_[u] = yd;
  s->pitch += pd;
  if (s->pitch > 30.0f) s->pitch = 30.0f;         // asymmetric view clamp
  if (s->pitch < -70.0f) s->pitch = -70.0f;
  last_pd_[u] = pd;
  if (!s->base_vel_flag) {                        // moving-ground basevelocity fold
    float sc = static_cast<float>(cfg_.phys.msec * 0.001) * 0.5f + 1.0f;
    for (int k = 0; k < 3; ++k) s->velocity[k] += sc * s->basevelocity[k];
    s->basevelocity[0] = s->basevelocity[1] = s->basevelocity[2] = 0.0f;
  }
  s->base_vel_flag = 0;
  goal_hit_[u] = 0;
  forced = forced || pending_fail_[u];
  pending_fail_[u] = 0;
  float prev_org[3];
  copy3(prev_org, s->origin);
  float prev_prog = s->progress;
  // View pitch never enters the movement tick (it aims the sensor only).
  MoveResult mr = mover_.tick(s, &memo_[u], s->yaw, 0.0f, fmove, smove, buttons, cfg_.phys.msec);
  s->tick++;
  bool fail = false, complete = false;
  if (goal_on_) {
    const int uh = (cfg_.phys.enable_duck && s->ducked) ? 1 : 0;
    float lo[3], hi[3];
    for (int k = 0; k < 3; ++k) { lo[k] = goal_min_[k] - kPlayerMaxs[uh][k]; hi[k] = goal_max_[k] - kPlayerMins[uh][k]; }
    if (segment_hits_box(prev_org, s->origin, lo, hi)) { complete = true; goal_hit_[u] = 1; }
  }
  int trig = complete ? 0 : apply_triggers(i, s);
  if (trig == 1) fail = true;
  if (trig == 2 && teleport_fail_) fail = true;
  if (forced && !complete) fail = true;
  float r = 0;
  const int nwp = static_cast<int>(wp_.size() / 3);
  if (nwp >= 2) {
    s->progress = spline_project(s->origin, &s->seg_hint);
    if (trig != 2) r = 0.05f * (s->progress - prev_prog);
    if (s->progress > s->best_progress) s->best_progress = s->progress;
    if (s->progress >= total_len_ - 50.0f) {
      const float* fin = &wp_[3 * static_cast<size_t>(nwp - 1)];
      float dx = s->origin[0] - fin[0], dy = s->origin[1] - fin[1], dz = s->origin[2] - fin[2];
      if (dx * dx + dy * dy + dz * dz < 150.0f * 150.0f) { complete = true; r += 50.0f; }
    }
  }
  if (mr.waterlevel >= 2 && cfg_.water_fail) fail = true;
  if (s->origin[2] < kill_z_) fail = true;
  s->stuck_ticks = mr.blocked ? s->stuck_ticks + 1 : 0;
  if (s->stuck_ticks >= 5) fail = true;
  bool truncated = s->tick >= cfg_.max_episode_ticks;
  bool d = fail || complete;
  TickOut out{r, d, truncated && !d, complete};
  if (d || truncated) {
    if (term_row) write_obs(*s, last_yd_[u], last_pd_[u], term_row);
    if (term_rec) {
      copy3(term_rec + kTermOrigin, s->origin);
      term_rec[kTermYaw] = s->yaw;
      term_rec[kTermPitch] = s->pitch;
      term_rec[kTermDucked] = static_cast<float>(s->ducked);
      term_rec[kTermTick] = static_cast<float>(s->tick);
    }
    reset_env(i);
    if (obs_row) write_obs(st_[u], 0.0f, 0.0f, obs_row);
  } else if (obs_row) {
    write_obs(*s, last_yd_[u], last_pd_[u], obs_row);
  }
  return out;
}

void EnvBatch::reset_all(uint64_t seed, float* obs) {
  for (int i = 0; i < cfg_.num_envs; ++i) {
    uint64_t t = seed + static_cast<uint64_t>(i);      // per-env stream through the mixer
    rng_[static_cast<size_t>(i)] = splitmix(&t) | 1;
    reset_env(i);
    if (obs) write_obs(st_[static_cast<size_t>(i)], 0.0f, 0.0f, &obs[static_cast<size_t>(i) * obs_dim_]);
  }
}

void EnvBatch::step(const int32_t* actions, float* obs, float* rewards, uint8_t* done, uint8_t* trunc,
                    float* terminal_obs) {
  pool_->run(cfg_.num_envs, [&](int b, int e) {
    for (int i = b; i < e; ++i) {
      const int32_t* a = &actions[static_cast<size_t>(i) * kActionDim];
      int yb = a[0] < 0 ? 0 : (a[0] > 14 ? 14 : a[0]);
      float yd = yaw_delta(st_[static_cast<size_t>(i)], yb);
      int pb = a[1] < 0 ? 0 : (a[1] > 6 ? 6 : a[1]);
      float pd = kPitchBins[pb] * (cfg_.pitch_rate_max_deg / 10.0f);
      float fm = a[2] <= 0 ? -400.0f : (a[2] >= 2 ? 400.0f : 0.0f);
      float sm = a[3] <= 0 ? -400.0f : (a[3] >= 2 ? 400.0f : 0.0f);
      int buttons = (a[4] ? kInJump : 0) | (a[5] ? kInDuck : 0);
      float* orow = &obs[static_cast<size_t>(i) * obs_dim_];
      float* trow = &terminal_obs[static_cast<size_t>(i) * obs_dim_];
      TickOut t = tick_env(i, yd, pd, fm, sm, buttons, false, orow, trow, nullptr);
      rewards[i] = t.reward;
      done[i] = t.done ? 1 : 0;
      trunc[i] = t.trunc ? 1 : 0;
    }
  });
}

void EnvBatch::step_k(const int32_t* actions, int action_stride, int yaw_slot, int fail_slot, int k, RowOut obs,
                      RowOut term_obs, RowOut rec, RowOut term_rec) {
  step_k_range(0, cfg_.num_envs, actions, action_stride, yaw_slot, fail_slot, k, obs, term_obs, rec, term_rec);
}

void EnvBatch::step_k_range(int lo, int hi, const int32_t* actions, int action_stride, int yaw_slot, int fail_slot,
                            int k, RowOut obs, RowOut term_obs, RowOut rec, RowOut term_rec) {
  if (k < 1) k = 1;
  lo = lo < 0 ? 0 : lo;
  hi = hi > cfg_.num_envs ? cfg_.num_envs : hi;
  if (hi <= lo) return;
  pool_->run(hi - lo, [&](int b, int e) {
    for (int i = b + lo; i < e + lo; ++i) {
      const int32_t* a = &actions[static_cast<size_t>(i) * static_cast<size_t>(action_stride)];
      int pb = a[1] < 0 ? 0 : (a[1] > 6 ? 6 : a[1]);
      float pd = kPitchBins[pb] * (cfg_.pitch_rate_max_deg / 10.0f);
      float fm = a[2] <= 0 ? -400.0f : (a[2] >= 2 ? 400.0f : 0.0f);
      float sm = a[3] <= 0 ? -400.0f : (a[3] >= 2 ? 400.0f : 0.0f);
      int buttons = (a[4] ? kInJump : 0) | (a[5] ? kInDuck : 0);
      int yb = a[0] < 0 ? 0 : (a[0] > 14 ? 14 : a[0]);
      float yc = 0.f;
      if (yaw_slot >= 0) {
        std::memcpy(&yc, &a[yaw_slot], sizeof yc);
        yc = yc > 1.f ? 1.f : (yc < -1.f ? -1.f : yc);
        if (yc != yc) yc = 0.f;
      }
      bool forced = fail_slot >= 0 && a[fail_slot] != 0;
      float rsum = 0;
      bool done = false, trunc = false, goal = false;
      for (int j = 0; j < k; ++j) {
        float yd = yaw_slot >= 0 ? yc * cfg_.yaw_rate_max_deg : yaw_delta(st_[static_cast<size_t>(i)], yb);
        float* orow = (j == k - 1 && obs.ptr) ? obs.row(i) : nullptr;
        TickOut t = tick_env(i, yd, pd, fm, sm, buttons, forced && j == 0, orow,
                             term_obs.ptr ? term_obs.row(i) : nullptr, term_rec.ptr ? term_rec.row(i) : nullptr);
        rsum += t.reward;
        done |= t.done;
        trunc |= t.trunc;
        goal |= t.goal;
      }
      if (rec.ptr) {
        const PlayerState& s = st_[static_cast<size_t>(i)];
        float* o = rec.row(i);
        copy3(o + kRecOrigin, s.origin);
        o[kRecYaw] = s.yaw;
        o[kRecPitch] = s.pitch;
        o[kRecDucked] = static_cast<float>(s.ducked);
        copy3(o + kRecVel, s.velocity);
        o[kRecTick] = static_cast<float>(s.tick);
        o[kRecReward] = rsum;
        o[kRecDone] = done ? 1.f : 0.f;
        o[kRecTrunc] = trunc ? 1.f : 0.f;
        o[kRecGoal] = goal ? 1.f : 0.f;
        o[kRecEnded] = (done || trunc) ? 1.f : 0.f;
        o[kRecOnground] = s.onground != -1 ? 1.f : 0.f;
      }
    }
  });
}

// ---- single-player primitives ------------------------------------------------
void EnvBatch::pm_step_usercmd(PlayerState* s, float yaw, float pitch, float fmove, float smove, int buttons, int msec) {
  if (msec > 50) {                                  // SV_RunCmd splits long commands
    int half = static_cast<int>(static_cast<uint8_t>(msec / 2.0));
    pm_step_usercmd(s, yaw, pitch, fmove, smove, buttons, half);
    pm_step_usercmd(s, yaw, pitch, fmove, smove, buttons, half);
    return;
  }
  float ft = static_cast<float>(msec * 0.001);
  if (!s->base_vel_flag) {
    float sc = ft * 0.5f + 1.0f;
    for (int k = 0; k < 3; ++k) s->velocity[k] += sc * s->basevelocity[k];
    s->basevelocity[0] = s->basevelocity[1] = s->basevelocity[2] = 0.0f;
  }
  s->base_vel_flag = 0;
  mover_.tick(s, &single_memo_, yaw, pitch, fmove, smove, buttons, msec);
  s->tick++;
}

int EnvBatch::play_step(PlayerState* s, float yaw, float pitch, float fmove, float smove, int buttons, int msec) {
  if (msec > 50) {
    int half = static_cast<int>(static_cast<uint8_t>(msec / 2.0));
    int f = play_step(s, yaw, pitch, fmove, smove, buttons, half);
    return f | play_step(s, yaw, pitch, fmove, smove, buttons, half);
  }
  float ft = static_cast<float>(msec * 0.001);
  if (!s->base_vel_flag) {
    float sc = ft * 0.5f + 1.0f;
    for (int k = 0; k < 3; ++k) s->velocity[k] += sc * s->basevelocity[k];
    s->basevelocity[0] = s->basevelocity[1] = s->basevelocity[2] = 0.0f;
  }
  s->base_vel_flag = 0;
  MoveResult mr = mover_.tick(s, &single_memo_, yaw, pitch, fmove, smove, buttons, msec);
  s->tick++;
  // Live triggers on the caller's state, with env slot 0's push-once bookkeeping.
  int trig = apply_triggers(0, s);
  int flags = 0;
  if (trig == 2) flags |= 1;
  if (trig == 1) flags |= 2;
  if (mr.waterlevel >= 2) flags |= 4;
  if (mr.blocked) flags |= 8;
  return flags;
}

void EnvBatch::pm_step_single(PlayerState* s, const int32_t action[6]) {
  int yb = action[0] < 0 ? 0 : (action[0] > 14 ? 14 : action[0]);
  float yd = yaw_delta(*s, yb);
  int pb = action[1] < 0 ? 0 : (action[1] > 6 ? 6 : action[1]);
  float pd = kPitchBins[pb] * (cfg_.pitch_rate_max_deg / 10.0f);
  float fm = action[2] <= 0 ? -400.0f : (action[2] >= 2 ? 400.0f : 0.0f);
  float sm = action[3] <= 0 ? -400.0f : (action[3] >= 2 ? 400.0f : 0.0f);
  int buttons = (action[4] ? kInJump : 0) | (action[5] ? kInDuck : 0);
  s->yaw = wrap360(s->yaw + yd);
  s->pitch += pd;
  if (s->pitch > 30.0f) s->pitch = 30.0f;
  if (s->pitch < -70.0f) s->pitch = -70.0f;
  pm_step_usercmd(s, s->yaw, 0.0f, fm, sm, buttons, cfg_.phys.msec);
}

void EnvBatch::occupancy_grid(const float* mins, float cell, int nx, int ny, int nz, uint8_t* out) {
  pool_->run(nz, [&](int b, int e) {
    for (int iz = b; iz < e; ++iz)
      for (int iy = 0; iy < ny; ++iy)
        for (int ix = 0; ix < nx; ++ix) {
          float p[3] = {mins[0] + (ix + 0.5f) * cell, mins[1] + (iy + 0.5f) * cell, mins[2] + (iz + 0.5f) * cell};
          int pc = point_contents(*map_, p);
          bool solid = pc == kSolid || pc == kSky;
          if (!solid) {                          // solid brush entities too
            Trace tr;
            trace_player(*map_, 2, p, p, &tr);
            solid = tr.startsolid;
          }
          out[static_cast<size_t>(ix) + static_cast<size_t>(nx) * (static_cast<size_t>(iy) + static_cast<size_t>(ny) * static_cast<size_t>(iz))] = solid ? 1 : 0;
        }
  });
}

}  // namespace surf
