// gates.cpp — native acceptance gates of the simulator (a standalone executable).
//
// The reference ships C test programs run by its build script
// (tests/dump_map.c, test_trace.c, test_physics.c, bench.c); this executable
// restates their gates on a map it compiles itself with the BSP writer (a
// floor, a 50-degree surf ramp, a wall), so it needs no assets:
//   A  load: the compiled image loads, planes / clipnodes / models / spawns
//   B  traces: standing rest height over the floor, startsolid => fraction 0,
//      A->B / B->A agreement, point contents above / below the floor, the
//      ramp's face normal
//   C  physics: a standing player stays put, the jump apex matches
//      v0^2 / 2g, friction stops a walker, air acceleration is capped at 30
//      u/s of wish speed, a ramp slide with no input gains speed and never
//      touches ground
//   D  throughput: random actions through the env batch on one thread, no
//      NaN in any state, >= 100k env ticks/s
//   E  start-node grids: random traces and point contents starting at a grid
//      cell's node equal the root-started ones bit for bit (no reference
//      counterpart: the grids are this build's)
//   F  point-in-solid: player_point_solid equals the zero-length trace's
//      startsolid (this build's shortcut of PM_TestPlayerPosition)
// Exit status 0 when every gate passes; one line per check on stdout.
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <random>
#include <string>
#include <vector>

#include "../bspwrite.hpp"
#include "../collide.hpp"
#include "../env.hpp"
#include "../map.hpp"
#include "../movement.hpp"

using namespace surf;

namespace {

int g_fail = 0;

void check(bool ok, const char* what, double got = 0.0, double want = 0.0) {
  std::printf("%s %-56s got %.6g want %.6g\n", ok ? "PASS" : "FAIL", what, got, want);
  if (!ok) ++g_fail;
}

Brush box(float x0, float y0, float z0, float x1, float y1, float z1, int model = 0) {
  Brush b;
  b.model = model;
  b.planes = {{{1, 0, 0}, x1}, {{-1, 0, 0}, -x0}, {{0, 1, 0}, y1}, {{0, -1, 0}, -y0}, {{0, 0, 1}, z1},
              {{0, 0, -1}, -z0}};
  return b;
}

// wedge along x at y = cy: faces tilted `deg` from horizontal, base width w
Brush wedge(float x0, float x1, float cy, float w, float z0, float deg) {
  const float a = deg * 3.14159265358979f / 180.f, h = 0.5f * w * std::tan(a);
  Brush b;
  const float s = std::sin(a), c = std::cos(a);
  for (float side : {1.f, -1.f}) {
    BrushPlane p{{0.f, side * s, c}, 0.f};
    p.d = p.n[1] * (cy + side * 0.5f * w) + p.n[2] * z0;
    b.planes.push_back(p);
  }
  b.planes.push_back({{0, 0, -1}, -z0});
  b.planes.push_back({{1, 0, 0}, x1});
  b.planes.push_back({{-1, 0, 0}, -x0});
  (void)h;
  return b;
}

std::shared_ptr<Map> build_map() {
  BspWriter w;
  w.add_brush(box(-4096, -4096, -16, 4096, 4096, 0));          // floor
  w.add_brush(box(3000, -4096, 0, 3100, 4096, 1024));          // wall
  w.add_brush(wedge(-2000, 2000, 1500, 800, 0, 50));            // surf ramp along x
  w.set_entities(
      "{\n\"classname\" \"worldspawn\"\n}\n{\n\"classname\" \"info_player_start\"\n\"origin\" \"0 0 64\"\n"
      "\"angle\" \"0\"\n}\n");
  std::vector<uint8_t> img;
  std::string err;
  if (!w.build(&img, &err)) {
    std::printf("FAIL bsp write: %s\n", err.c_str());
    return nullptr;
  }
  auto m = std::make_shared<Map>();
  if (!m->load_memory(img.data(), img.size(), &err)) {
    std::printf("FAIL bsp load: %s\n", err.c_str());
    return nullptr;
  }
  return m;
}

float hspeed(const PlayerState& s) { return std::hypot(s.velocity[0], s.velocity[1]); }

PlayerState spawn(float x, float y, float z) {
  PlayerState s;
  std::memset(&s, 0, sizeof s);
  s.origin[0] = x;
  s.origin[1] = y;
  s.origin[2] = z;
  s.onground = -1;
  return s;
}

}  // namespace

int main() {
  auto map = build_map();
  if (!map) return 2;
  // ---- A: load
  check(!map->planes.empty(), "A planes present", static_cast<double>(map->planes.size()), 1);
  check(!map->clipnodes.empty(), "A clipnodes present", static_cast<double>(map->clipnodes.size()), 1);
  check(map->spawns.size() == 1, "A one spawn point", static_cast<double>(map->spawns.size()), 1);

  // ---- B: traces (usehull 0 = standing player box, mins z -36)
  {
    Trace tr;
    const float a[3] = {0, 0, 200}, b[3] = {0, 0, -200};
    trace_player(*map, 0, a, b, &tr);
    check(std::fabs(tr.endpos[2] - 36.0f) < 0.1f, "B standing rest height above the floor", tr.endpos[2], 36.0);
    check(tr.normal[2] > 0.99f, "B floor normal points up", tr.normal[2], 1.0);
    Trace in;
    const float s[3] = {0, 0, -8}, e[3] = {0, 0, 100};
    trace_player(*map, 0, s, e, &in);
    check(in.startsolid && in.fraction == 0.0f, "B startsolid implies fraction 0", in.fraction, 0.0);
    Trace f1, f2;
    const float p[3] = {-500, -300, 300}, q[3] = {3500, -300, 300};
    trace_player(*map, 0, p, q, &f1);
    trace_player(*map, 0, q, p, &f2);
    const float hit1 = p[0] + f1.fraction * (q[0] - p[0]);
    const float hit2 = q[0] + f2.fraction * (p[0] - q[0]);
    check(std::fabs(hit1 - (3000.f - 16.f)) < 0.1f, "B wall stops the box at its near face", hit1, 2984.0);
    check(std::fabs(hit2 - (3100.f + 16.f)) < 0.1f, "B reverse trace stops at the far face", hit2, 3116.0);
    const float above[3] = {0, 0, 10}, below[3] = {0, 0, -8};
    check(point_contents(*map, above) == kEmpty, "B contents above the floor", point_contents(*map, above), kEmpty);
    check(point_contents(*map, below) == kSolid, "B contents inside the floor", point_contents(*map, below), kSolid);
    Trace r;
    const float ra[3] = {0, 1700, 2000}, rb[3] = {0, 1700, -100};
    trace_player(*map, 0, ra, rb, &r);
    const float nz = std::cos(50.f * 3.14159265f / 180.f);
    check(std::fabs(r.normal[2] - nz) < 1e-3f && r.normal[1] > 0.5f, "B ramp face normal", r.normal[2], nz);
  }

  // ---- C: physics
  Physics ph;
  ph.maxvelocity = 3500;
  PlayerMove pm(*map, ph);
  StuckMemo memo;
  {
    PlayerState s = spawn(0, 0, 37);
    for (int i = 0; i < 100; ++i) pm.tick(&s, &memo, 0, 0, 0, 0, 0, 10);
    check(hspeed(s) == 0.0f && std::fabs(s.origin[2] - 36.f) < 1.5f && s.onground != -1,
          "C standing player stays put", s.origin[2], 36.0);
  }
  {
    PlayerState s = spawn(0, 0, 37);
    for (int i = 0; i < 10; ++i) pm.tick(&s, &memo, 0, 0, 0, 0, 0, 10);
    const float z0 = s.origin[2];
    float top = z0;
    pm.tick(&s, &memo, 0, 0, 0, 0, 2 /*IN_JUMP*/, 10);
    for (int i = 0; i < 80; ++i) {
      pm.tick(&s, &memo, 0, 0, 0, 0, 0, 10);
      top = std::fmax(top, s.origin[2]);
    }
    const float v0 = std::sqrt(2.f * 800.f * 45.f);
    const float want = v0 * v0 / (2.f * 800.f);
    check(std::fabs((top - z0) - want) < 4.0f, "C jump apex ~ v0^2 / 2g", top - z0, want);
  }
  {
    PlayerState s = spawn(0, 0, 37);
    s.velocity[0] = 300;
    for (int i = 0; i < 200; ++i) pm.tick(&s, &memo, 0, 0, 0, 0, 0, 10);
    check(hspeed(s) == 0.0f, "C friction stops a sliding walker", hspeed(s), 0.0);
  }
  {
    // one airborne tick with sidemove perpendicular to the velocity: the
    // added speed is capped by the 30 u/s air wish speed
    PlayerState s = spawn(0, -2000, 600);
    s.velocity[0] = 600;
    const float before = hspeed(s);
    pm.tick(&s, &memo, 0, 0, 0, 400, 0, 10);
    const float gain = std::fabs(s.velocity[1]);
    check(gain <= 30.0f + 1e-3f && gain > 0.0f, "C air acceleration capped at 30 u/s", gain, 30.0);
    (void)before;
  }
  {
    // drop onto the ramp face, no input: slides and gains speed, never grounded
    PlayerState s = spawn(0, 1700, 700);
    bool grounded = false;
    float v_start = -1;
    for (int i = 0; i < 150; ++i) {
      pm.tick(&s, &memo, 0, 0, 0, 0, 0, 10);
      if (i == 60) v_start = hspeed(s);
      grounded |= s.onground != -1 && s.origin[2] > 40.f;
    }
    check(!grounded && hspeed(s) > v_start + 50.f, "C ramp slide gains speed without ground", hspeed(s), v_start);
  }

  // ---- D: throughput on one thread
  {
    EnvConfig cfg;
    cfg.num_envs = 256;
    cfg.spawn_mode = 0;
    cfg.phys.maxvelocity = 3500;
    EnvBatch env(map, cfg, 1);
    std::vector<float> obs(static_cast<size_t>(cfg.num_envs) * env.obs_dim()), term(obs.size());
    std::vector<float> rew(cfg.num_envs);
    std::vector<uint8_t> done(cfg.num_envs), trunc(cfg.num_envs);
    std::vector<int32_t> act(static_cast<size_t>(cfg.num_envs) * 6);
    env.reset_all(7, obs.data());
    std::mt19937 rng(5);
    const int nvec[6] = {15, 7, 3, 3, 2, 2};
    const int ticks = 600;
    const auto t0 = std::chrono::steady_clock::now();
    bool finite = true;
    for (int t = 0; t < ticks; ++t) {
      for (size_t i = 0; i < act.size(); ++i) act[i] = static_cast<int32_t>(rng() % nvec[i % 6]);
      env.step(act.data(), obs.data(), rew.data(), done.data(), trunc.data(), term.data());
      for (float v : obs) finite &= std::isfinite(v);
    }
    const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    const double rate = static_cast<double>(ticks) * cfg.num_envs / dt;
    check(finite, "D no NaN / inf in any observation", finite ? 1 : 0, 1);
    check(rate >= 1e5, "D single-thread env ticks/s", rate, 1e5);
  }
  // ---- E: start-node grids: traces and point contents that start at a grid
  // cell's node equal those that start at the root, bit for bit
  {
    const MapView with = map->view();
    MapView without = with;
    for (auto& g : without.world_grid) g = HullGrid();
    std::mt19937 rng(11);
    std::uniform_real_distribution<float> ux(with.world_mins[0] - 40, with.world_maxs[0] + 40),
        uy(with.world_mins[1] - 40, with.world_maxs[1] + 40), uz(with.world_mins[2] - 40, with.world_maxs[2] + 40);
    std::uniform_real_distribution<float> step(-40.f, 40.f);
    int mismatch = 0, from_grid = 0;
    const int n = 200000;
    for (int i = 0; i < n; ++i) {
      const float a[3] = {ux(rng), uy(rng), uz(rng)};
      // short moves (most pmove traces) and long ones
      const float sc = i % 4 == 0 ? 20.f : 1.f;
      const float b[3] = {a[0] + sc * step(rng), a[1] + sc * step(rng), a[2] + sc * step(rng)};
      const int usehull = i % 3;
      Trace t1, t2;
      trace_player(with, usehull, a, b, &t1);
      trace_player(without, usehull, a, b, &t2);
      const HullView hv = with.hull(0, bsp_hull_of_usehull(usehull));
      float la[3], lb[3];
      for (int k = 0; k < 3; ++k) {
        const float off = hv.clip_mins[k] - player_mins(usehull, k) + with.models[0].origin[k];
        la[k] = a[k] - off;
        lb[k] = b[k] - off;
      }
      from_grid += hv.grid.segment_start(la, lb) != HullGrid::kNone;
      if (std::memcmp(&t1, &t2, sizeof t1) != 0) ++mismatch;
      if (point_contents(with, a) != point_contents(without, a)) ++mismatch;
    }
    check(mismatch == 0, "E grid-started traces / contents == root-started", mismatch, 0);
    check(from_grid > n / 4, "E grid starts most short traces below the root", from_grid, n / 4);
  }
  // ---- F: the point-in-solid test (stuck checks, unduck headroom) answers as
  // the zero-length trace's startsolid, with and without grids, at random
  // points and at trace end points (boxes resting against a surface)
  {
    const MapView with = map->view();
    MapView without = with;
    for (auto& g : without.world_grid) g = HullGrid();
    std::mt19937 rng(13);
    std::uniform_real_distribution<float> ux(with.world_mins[0] - 40, with.world_maxs[0] + 40),
        uy(with.world_mins[1] - 40, with.world_maxs[1] + 40), uz(with.world_mins[2] - 40, with.world_maxs[2] + 40);
    std::uniform_real_distribution<float> step(-200.f, 200.f);
    int mismatch = 0, solid = 0;
    const int n = 200000;
    for (int i = 0; i < n; ++i) {
      const int usehull = i % 3;
      float p[3] = {ux(rng), uy(rng), uz(rng)};
      if (i % 2) {                        // the end of a sweep: resting against whatever it hit
        const float b[3] = {p[0] + step(rng), p[1] + step(rng), p[2] + step(rng)};
        Trace t;
        trace_player(with, usehull, p, b, &t);
        for (int k = 0; k < 3; ++k) p[k] = t.endpos[k];
      }
      Trace tw, to;
      trace_player(with, usehull, p, p, &tw);
      trace_player(without, usehull, p, p, &to);
      const bool fw = player_point_solid(with, usehull, p), fo = player_point_solid(without, usehull, p);
      mismatch += (fw != tw.startsolid) + (fo != to.startsolid);
      solid += fw;
    }
    check(mismatch == 0, "F point-in-solid == zero-length trace startsolid", mismatch, 0);
    check(solid > n / 20 && solid < n - n / 20, "F both answers occur", solid, n / 2);
  }
  std::printf("%s: %d failed\n", g_fail ? "FAILED" : "OK", g_fail);
  return g_fail ? 1 : 0;
}
