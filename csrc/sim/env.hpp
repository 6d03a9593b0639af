// env.hpp — vectorized surf environment over PlayerMove.
//
// Behaviour matches the reference batch env (src/env.c:529-644): action
// decode, basevelocity fold, one pm tick, swept goal-box test, post-move
// triggers, fail rules, spline progress reward and same-step autoreset with a
// terminal observation. On top of that:
//   * step_k fuses K physics ticks (action repeat) into one call and reduces
//     the per-tick signals (reward sum, done/trunc/goal OR) in C++;
//   * outputs land in caller rows of arbitrary stride, so Python can hand in
//     one pinned host buffer and ship it to the GPU with a single async copy;
//   * a continuous yaw action (degrees-per-tick fraction in [-1, 1]) may
//     replace the discrete yaw bin;
//   * a persistent thread pool replaces the per-call OpenMP team;
//   * the per-env rules live in env_core.hpp (EnvCore, host + device code):
//     this class owns the host arrays and runs EnvCore over them, the GPU env
//     (csrc/kernels/env_gpu.cu) runs the same EnvCore over device copies.
#pragma once
#include <cstdint>
#include <memory>
#include <vector>

#include "env_core.hpp"
#include "thread_pool.hpp"

namespace surf {

class EnvBatch {
 public:
  EnvBatch(std::shared_ptr<const Map> map, const EnvConfig& cfg, int threads);
  ~EnvBatch() { step_wait(); }            // no worker may outlive the arrays it steps
  EnvBatch(const EnvBatch&) = delete;
  EnvBatch& operator=(const EnvBatch&) = delete;
  int obs_dim() const { return obs_dim_; }
  int num_envs() const { return cfg_.num_envs; }
  const EnvConfig& config() const { return cfg_; }
  const Map& map() const { return *map_; }

  int set_waypoints(const float* xyz, int count);
  int set_spawn_pool(const PlayerState* pool, int n);
  void set_teleport_fail(bool on) { teleport_fail_ = on; sync_core(); }
  void set_goal_box(const float* mins, const float* maxs);
  void force_fail(const uint8_t* mask);
  const uint8_t* goal_hits() const { return goal_hit_.data(); }

  void reset_all(uint64_t seed, float* obs);
  // One tick for every env (reference-compatible contract).
  void step(const int32_t* actions, float* obs, float* rewards, uint8_t* done, uint8_t* trunc, float* terminal_obs);
  // K ticks of action repeat. actions: int32 rows of `action_stride` (slots
  // 0..5 the discrete action); yaw_slot >= 0: that slot holds a float in
  // [-1, 1] (bit pattern) replacing the yaw bin; fail_slot >= 0: a non-zero
  // value there force-fails the env on the first tick (stall kill).
  void step_k(const int32_t* actions, int action_stride, int yaw_slot, int fail_slot, int k, RowOut obs,
              RowOut term_obs, RowOut rec, RowOut term_rec);
  // step_k over envs [lo, hi) only (pointers still index the whole batch), so
  // that two halves of the batch can alternate with the GPU work of the other.
  void step_k_range(int lo, int hi, const int32_t* actions, int action_stride, int yaw_slot, int fail_slot, int k,
                    RowOut obs, RowOut term_obs, RowOut rec, RowOut term_rec);
  // step_k_range on the pool's workers: returns at once; step_wait() joins
  // the work and returns when it is done. The action and row buffers must
  // stay untouched (for the envs of the range) until then, and no other
  // batch call may come in between except step_wait(). Every other entry
  // point waits first.
  void step_k_range_async(int lo, int hi, const int32_t* actions, int action_stride, int yaw_slot, int fail_slot,
                          int k, RowOut obs, RowOut term_obs, RowOut rec, RowOut term_rec);
  void step_wait();
  // The order the last step of [lo, hi) visited its envs (Morton order of
  // their x-y cells), as offsets from lo: out[j] = env - lo. The identity
  // before that range's first step. Also the order a camera should render
  // them in (neighbours share cached map data there too).
  void env_order(int lo, int hi, int32_t* out) const;

  PlayerState* states() { return st_.data(); }
  void set_state(int env, const PlayerState& s);

  // Single-player primitives (parity harness, spawn auditions, play client).
  void pm_step_usercmd(PlayerState* st, float yaw, float pitch, float fmove, float smove, int buttons, int msec);
  int play_step(PlayerState* st, float yaw, float pitch, float fmove, float smove, int buttons, int msec);
  void pm_step_single(PlayerState* st, const int32_t action[6]);
  void occupancy_grid(const float* mins, float cell, int nx, int ny, int nz, uint8_t* out);

 // The EnvCore over this batch's arrays (rebuilt whenever an array changes).
  const EnvCore& core() const { return core_; }
  const std::vector<float>& waypoints() const { return wp_; }
  const std::vector<float>& cumulative() const { return cum_; }
  const std::vector<float>& tangents() const { return tang_; }
  const std::vector<float>& teleport_progress() const { return tele_progress_; }
  const std::vector<PlayerState>& spawn_pool() const { return spawn_pool_; }

 private:
  void sync_core();
  void write_lidar(const PlayerState& s, float* o) const;
  // The order step_k_range visits envs [lo, hi) in: Morton order of their
  // x-y cells, rebuilt every kOrderEvery calls for that range. Neighbouring
  // envs share clip-tree and start-grid cache lines; no env's result depends
  // on the order (each env owns its state, memos and random stream).
  const int32_t* spatial_order(int lo, int hi);
  struct RangeOrder {
    int lo = 0, hi = 0, age = 0;
    std::vector<int32_t> idx;
  };
  std::vector<RangeOrder> orders_;
  bool in_flight_ = false;               // a step_k_range_async job not yet waited for

  std::shared_ptr<const Map> map_;
  EnvConfig cfg_;
  std::unique_ptr<ThreadPool> pool_;
  int obs_dim_ = kObsFixed;
  float kill_z_ = 0, map_center_[3] = {0, 0, 0};
  std::vector<float> wp_, cum_, tang_;   // progress spline
  float total_len_ = 0;
  std::vector<float> tele_progress_;     // teleport destination progress per trigger
  std::vector<PlayerState> spawn_pool_;
  bool teleport_fail_ = false;
  bool goal_on_ = false;
  float goal_min_[3] = {0, 0, 0}, goal_max_[3] = {0, 0, 0};
  std::vector<PlayerState> st_;
  std::vector<StuckMemo> memo_;
  std::vector<GroundMemo> ground_;
  std::vector<float> last_yd_, last_pd_;
  std::vector<uint64_t> rng_;
  std::vector<uint64_t> push_used_;      // per env: bitset over triggers
  int push_words_ = 1;
  std::vector<uint8_t> goal_hit_, pending_fail_;
  StuckMemo single_memo_;
  EnvCore core_;
};

}  // namespace surf
