// env.cpp — vectorized env. See env.hpp.
#include "env.hpp"

#include <algorithm>

#include <cmath>
#include <cstring>

namespace surf {
namespace {
constexpr double kPiD = 3.14159265358979323846;
inline void copy3(float* d, const float* s) { d[0] = s[0]; d[1] = s[1]; d[2] = s[2]; }
template <typename T>
Span<T> span_of(const std::vector<T>& v) {
  Span<T> s;
  s.p = v.data();
  s.n = static_cast<int32_t>(v.size());
  return s;
}
}  // namespace

EnvBatch::EnvBatch(std::shared_ptr<const Map> map, const EnvConfig& cfg, int threads)
    : map_(std::move(map)), cfg_(cfg) {
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
  ground_.assign(n, GroundMemo{});
  last_yd_.assign(n, 0.f);
  last_pd_.assign(n, 0.f);
  rng_.assign(n, 0);
  push_words_ = static_cast<int>((map_->triggers.size() + 63) / 64);
  if (push_words_ < 1) push_words_ = 1;
  push_used_.assign(n * static_cast<size_t>(push_words_), 0);
  goal_hit_.assign(n, 0);
  pending_fail_.assign(n, 0);
  pool_ = std::make_unique<ThreadPool>(threads);
  sync_core();
}

void EnvBatch::sync_core() {
  EnvCore& c = core_;
  c.cfg = cfg_;
  c.map = map_->view();
  c.mover = PlayerMove(c.map, cfg_.phys);
  c.kill_z = kill_z_;
  copy3(c.map_center, map_center_);
  c.wp = span_of(wp_);
  c.cum = span_of(cum_);
  c.tang = span_of(tang_);
  c.tele_progress = span_of(tele_progress_);
  c.total_len = total_len_;
  c.spawn_pool = span_of(spawn_pool_);
  c.teleport_fail = teleport_fail_ ? 1 : 0;
  c.goal_on = goal_on_ ? 1 : 0;
  copy3(c.goal_min, goal_min_);
  copy3(c.goal_max, goal_max_);
  c.st = st_.data();
  c.memo = memo_.data();
  c.ground = ground_.data();
  c.last_yd = last_yd_.data();
  c.last_pd = last_pd_.data();
  c.rng = rng_.data();
  c.push_used = push_used_.data();
  c.push_words = push_words_;
  c.goal_hit = goal_hit_.data();
  c.pending_fail = pending_fail_.data();
}

int EnvBatch::set_waypoints(const float* xyz, int count) {
  step_wait();
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
  sync_core();
  for (PlayerState& s : st_) {
    if (s.seg_hint < 0) s.seg_hint = 0;
    if (s.seg_hint > count - 2) s.seg_hint = count - 2;
    s.progress = core_.spline_project(s.origin, &s.seg_hint);
    if (s.best_progress > total_len_) s.best_progress = s.progress;
  }
  return 0;
}

int EnvBatch::set_spawn_pool(const PlayerState* pool, int n) {
  step_wait();
  if (!pool || n < 1) return -1;
  spawn_pool_.assign(pool, pool + n);
  sync_core();
  return 0;
}

void EnvBatch::set_goal_box(const float* mins, const float* maxs) {
  step_wait();
  if (!mins || !maxs) {
    goal_on_ = false;
  } else {
    copy3(goal_min_, mins);
    copy3(goal_max_, maxs);
    goal_on_ = true;
  }
  sync_core();
}

void EnvBatch::force_fail(const uint8_t* mask) {
  step_wait();
  if (!mask) return;
  for (int i = 0; i < cfg_.num_envs; ++i)
    if (mask[i]) pending_fail_[static_cast<size_t>(i)] = 1;
}

void EnvBatch::set_state(int env, const PlayerState& s) {
  step_wait();
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

void EnvBatch::reset_all(uint64_t seed, float* obs) {
  step_wait();
  for (int i = 0; i < cfg_.num_envs; ++i) {
    core_.seed_and_reset(i, seed);
    if (obs) {
      float* o = &obs[static_cast<size_t>(i) * obs_dim_];
      core_.write_obs(st_[static_cast<size_t>(i)], 0.0f, 0.0f, o);
      write_lidar(st_[static_cast<size_t>(i)], o + kObsFixed);
    }
  }
}

void EnvBatch::step(const int32_t* actions, float* obs, float* rewards, uint8_t* done, uint8_t* trunc,
                    float* terminal_obs) {
  step_wait();
  auto lidar = [this](const PlayerState& s, float* o) { write_lidar(s, o); };
  pool_->run(cfg_.num_envs, [&](int b, int e) {
    for (int i = b; i < e; ++i) {
      const int32_t* a = &actions[static_cast<size_t>(i) * kActionDim];
      int yb = a[0] < 0 ? 0 : (a[0] > 14 ? 14 : a[0]);
      float yd = core_.yaw_delta(st_[static_cast<size_t>(i)], yb);
      int pb = a[1] < 0 ? 0 : (a[1] > 6 ? 6 : a[1]);
      float pd = envk::pitch_bin(pb) * (cfg_.pitch_rate_max_deg / 10.0f);
      float fm = a[2] <= 0 ? -400.0f : (a[2] >= 2 ? 400.0f : 0.0f);
      float sm = a[3] <= 0 ? -400.0f : (a[3] >= 2 ? 400.0f : 0.0f);
      int buttons = (a[4] ? kInJump : 0) | (a[5] ? kInDuck : 0);
      float* orow = &obs[static_cast<size_t>(i) * obs_dim_];
      float* trow = &terminal_obs[static_cast<size_t>(i) * obs_dim_];
      EnvCore::TickOut t = core_.tick_env(i, yd, pd, fm, sm, buttons, false, orow, trow, nullptr, lidar);
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
  step_k_range_async(lo, hi, actions, action_stride, yaw_slot, fail_slot, k, obs, term_obs, rec, term_rec);
  step_wait();
}

void EnvBatch::step_k_range_async(int lo, int hi, const int32_t* actions, int action_stride, int yaw_slot,
                                  int fail_slot, int k, RowOut obs, RowOut term_obs, RowOut rec, RowOut term_rec) {
  step_wait();                            // one job in flight at a time
  if (k < 1) k = 1;
  lo = lo < 0 ? 0 : lo;
  hi = hi > cfg_.num_envs ? cfg_.num_envs : hi;
  if (hi <= lo) return;
  const int32_t* order = spatial_order(lo, hi);
  const EnvCore* core = &core_;
  const EnvBatch* self = this;
  pool_->run_async(hi - lo, [=](int b, int e) {
    auto lidar = [self](const PlayerState& s, float* o) { self->write_lidar(s, o); };
    for (int j = b; j < e; ++j) {
      const int i = order[j];
      const int32_t* a = &actions[static_cast<size_t>(i) * static_cast<size_t>(action_stride)];
      core->step_k_one(i, a, yaw_slot, fail_slot, k, obs, term_obs, rec, term_rec, lidar);
    }
  });
  in_flight_ = true;
}

void EnvBatch::step_wait() {
  if (!in_flight_) return;
  pool_->wait();
  in_flight_ = false;
}

void EnvBatch::env_order(int lo, int hi, int32_t* out) const {
  for (const RangeOrder& o : orders_) {
    if (o.lo == lo && o.hi == hi && static_cast<int>(o.idx.size()) == hi - lo) {
      for (int j = 0; j < hi - lo; ++j) out[j] = o.idx[static_cast<size_t>(j)] - lo;
      return;
    }
  }
  for (int j = 0; j < hi - lo; ++j) out[j] = j;
}

const int32_t* EnvBatch::spatial_order(int lo, int hi) {
  constexpr int kOrderEvery = 8;          // calls between re-sorts (players move ~100u per call)
  constexpr float kCell = 256.f;          // Morton cell edge (units)
  RangeOrder* r = nullptr;
  for (RangeOrder& o : orders_)
    if (o.lo == lo && o.hi == hi) r = &o;
  if (!r) {
    orders_.push_back(RangeOrder{lo, hi, kOrderEvery, {}});
    r = &orders_.back();
  }
  if (r->age++ < kOrderEvery) return r->idx.data();
  r->age = 1;
  std::vector<std::pair<uint32_t, int32_t>> key(static_cast<size_t>(hi - lo));
  for (int i = lo; i < hi; ++i) {
    uint32_t c[2];
    for (int a = 0; a < 2; ++a) {
      const float f = (st_[static_cast<size_t>(i)].origin[a] - map_->world_mins[a]) / kCell;
      c[a] = f > 0.f ? (f < 1023.f ? static_cast<uint32_t>(f) : 1023u) : 0u;   // NaN -> 0
    }
    uint32_t m = 0;
    for (int bit = 0; bit < 10; ++bit) m |= ((c[0] >> bit) & 1u) << (2 * bit) | ((c[1] >> bit) & 1u) << (2 * bit + 1);
    key[static_cast<size_t>(i - lo)] = {m, i};
  }
  std::sort(key.begin(), key.end());
  r->idx.resize(key.size());
  for (size_t j = 0; j < key.size(); ++j) r->idx[j] = key[j].second;
  return r->idx.data();
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
  core_.mover.tick(s, &single_memo_, yaw, pitch, fmove, smove, buttons, msec);
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
  MoveResult mr = core_.mover.tick(s, &single_memo_, yaw, pitch, fmove, smove, buttons, msec);
  s->tick++;
  // Live triggers on the caller's state, with env slot 0's push-once bookkeeping.
  int trig = core_.apply_triggers(0, s);
  int flags = 0;
  if (trig == 2) flags |= 1;
  if (trig == 1) flags |= 2;
  if (mr.waterlevel >= 2) flags |= 4;
  if (mr.blocked) flags |= 8;
  return flags;
}

void EnvBatch::pm_step_single(PlayerState* s, const int32_t action[6]) {
  int yb = action[0] < 0 ? 0 : (action[0] > 14 ? 14 : action[0]);
  float yd = core_.yaw_delta(*s, yb);
  int pb = action[1] < 0 ? 0 : (action[1] > 6 ? 6 : action[1]);
  float pd = envk::pitch_bin(pb) * (cfg_.pitch_rate_max_deg / 10.0f);
  float fm = action[2] <= 0 ? -400.0f : (action[2] >= 2 ? 400.0f : 0.0f);
  float sm = action[3] <= 0 ? -400.0f : (action[3] >= 2 ? 400.0f : 0.0f);
  int buttons = (action[4] ? kInJump : 0) | (action[5] ? kInDuck : 0);
  s->yaw = envk::wrap360(s->yaw + yd);
  s->pitch += pd;
  if (s->pitch > 30.0f) s->pitch = 30.0f;
  if (s->pitch < -70.0f) s->pitch = -70.0f;
  pm_step_usercmd(s, s->yaw, 0.0f, fm, sm, buttons, cfg_.phys.msec);
}

void EnvBatch::occupancy_grid(const float* mins, float cell, int nx, int ny, int nz, uint8_t* out) {
  step_wait();
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
