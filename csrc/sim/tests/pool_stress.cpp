// pool_stress.cpp — the env batch's worker pool under a thread sanitizer.
//
// The same seed and actions are stepped through one env batch with 1 worker
// thread and one with 4 (step_k with K = 3; the 4-thread batch in two groups
// through step_k_range_async / step_wait, episodes short enough that most
// envs autoreset several times); every player state and every output row
// must be identical. Built with -fsanitize=thread (tests/test_sanitizers.py),
// any data race between the workers and the caller is reported and fails the
// run. The reference has no sanitizer runs (its safety net is determinism
// flags and a NaN scan); this executable has no reference counterpart.
// Exit status 0 when the batches agree.
#include <cstdio>
#include <cstring>
#include <memory>
#include <random>
#include <string>
#include <vector>

#include "../bspwrite.hpp"
#include "../env.hpp"
#include "../map.hpp"

using namespace surf;

namespace {

Brush box(float x0, float y0, float z0, float x1, float y1, float z1) {
  Brush b;
  b.planes = {{{1, 0, 0}, x1}, {{-1, 0, 0}, -x0}, {{0, 1, 0}, y1}, {{0, -1, 0}, -y0}, {{0, 0, 1}, z1}, {{0, 0, -1}, -z0}};
  return b;
}

std::shared_ptr<Map> build_map() {
  BspWriter w;
  w.add_brush(box(-2048, -2048, -16, 2048, 2048, 0));        // floor
  w.add_brush(box(1500, -2048, 0, 1600, 2048, 512));         // wall
  w.add_brush(box(-600, -200, 0, -400, 200, 96));            // a block to walk into
  w.set_entities(
      "{\n\"classname\" \"worldspawn\"\n}\n{\n\"classname\" \"info_player_start\"\n\"origin\" \"0 0 64\"\n"
      "\"angle\" \"0\"\n}\n{\n\"classname\" \"info_player_start\"\n\"origin\" \"800 300 200\"\n\"angle\" \"90\"\n}\n");
  std::vector<uint8_t> img;
  std::string err;
  if (!w.build(&img, &err)) return nullptr;
  auto m = std::make_shared<Map>();
  if (!m->load_memory(img.data(), img.size(), &err)) return nullptr;
  return m;
}

}  // namespace

int main() {
  auto map = build_map();
  if (!map) {
    std::printf("FAIL map\n");
    return 2;
  }
  EnvConfig cfg;
  cfg.num_envs = 96;
  cfg.spawn_mode = 0;
  cfg.max_episode_ticks = 40;
  EnvBatch one(map, cfg, 1), four(map, cfg, 4);
  const int n = cfg.num_envs;
  std::vector<float> obs(static_cast<size_t>(n) * one.obs_dim());
  one.reset_all(9, obs.data());
  four.reset_all(9, obs.data());
  std::vector<float> o1(static_cast<size_t>(n) * 32), o4(o1.size()), t1(o1.size()), t4(o1.size());
  std::vector<float> r1(static_cast<size_t>(n) * kRecCols), r4(r1.size()), q1(static_cast<size_t>(n) * kTermCols),
      q4(q1.size());
  std::vector<int32_t> act(static_cast<size_t>(n) * 8, 0);
  std::mt19937 rng(3);
  const int nvec[6] = {15, 7, 3, 3, 2, 2};
  int bad = 0;
  for (int d = 0; d < 60; ++d) {
    for (int i = 0; i < n; ++i)
      for (int j = 0; j < 6; ++j) act[static_cast<size_t>(i) * 8 + j] = static_cast<int32_t>(rng() % nvec[j]);
    one.step_k(act.data(), 8, -1, -1, 3, RowOut{o1.data(), 32}, RowOut{t1.data(), 32}, RowOut{r1.data(), kRecCols},
               RowOut{q1.data(), kTermCols});
    // the 4-thread batch in two groups through the asynchronous entry point,
    // the caller reading the first group's rows while the second steps
    four.step_k_range_async(0, 40, act.data(), 8, -1, -1, 3, RowOut{o4.data(), 32}, RowOut{t4.data(), 32},
                            RowOut{r4.data(), kRecCols}, RowOut{q4.data(), kTermCols});
    four.step_wait();
    four.step_k_range_async(40, n, act.data(), 8, -1, -1, 3, RowOut{o4.data(), 32}, RowOut{t4.data(), 32},
                            RowOut{r4.data(), kRecCols}, RowOut{q4.data(), kTermCols});
    float first = 0;
    for (int i = 0; i < 40; ++i) first += r4[static_cast<size_t>(i) * kRecCols];
    four.step_wait();
    if (first != first) ++bad;
    if (std::memcmp(one.states(), four.states(), sizeof(PlayerState) * n) != 0 || o1 != o4 || r1 != r4 || q1 != q4)
      ++bad;
  }
  std::printf("%s: %d of 60 decisions differ between 1 and 4 worker threads\n", bad ? "FAIL" : "OK", bad);
  return bad ? 1 : 0;
}
