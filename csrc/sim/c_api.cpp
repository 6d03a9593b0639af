// c_api.cpp — the stable C ABI of the simulation library (libsurfsim.so).
//
// Python binds it with ctypes (calls release the GIL); the parity harness
// drives it side by side with the reference core. The state (108 B) and
// config (128 B) layouts match the reference's SurfState / SurfEnvConfig
// (src/surfcore.h:66-140), and the per-env functions mirror its exports
// (src/surfcore.h:155-234) under the `surfsim_` prefix.
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "bspwrite.hpp"
#include "env.hpp"
#include "mesh.hpp"

using namespace surf;

#define SURFSIM_API extern "C" __attribute__((visibility("default")))

namespace {
constexpr int32_t kAbiVersion = 1;

struct SimHandle {
  std::shared_ptr<Map> map;
  std::unique_ptr<EnvBatch> env;
};

void set_err(char* err, int len, const std::string& msg) {
  if (err && len > 0) {
    std::strncpy(err, msg.c_str(), static_cast<size_t>(len) - 1);
    err[len - 1] = 0;
  }
}

struct TraceOut {                   // SurfTrace-compatible (44 bytes)
  float endpos[3], normal[3], dist, fraction;
  int32_t startsolid, allsolid, ent;
};
static_assert(sizeof(TraceOut) == 44, "TraceOut layout");

SimHandle* make(std::shared_ptr<Map> map, const EnvConfig* cfg, int threads) {
  auto* h = new SimHandle;
  h->map = std::move(map);
  h->env = std::make_unique<EnvBatch>(h->map, *cfg, threads);
  return h;
}
}  // namespace

SURFSIM_API int32_t surfsim_abi_version() { return kAbiVersion; }
SURFSIM_API int32_t surfsim_sizeof_state() { return static_cast<int32_t>(sizeof(PlayerState)); }
SURFSIM_API int32_t surfsim_sizeof_config() { return static_cast<int32_t>(sizeof(EnvConfig)); }

SURFSIM_API void* surfsim_create(const char* path, const EnvConfig* cfg, int32_t threads, char* err, int32_t errlen) {
  auto map = std::make_shared<Map>();
  std::string e;
  if (!map->load_file(path, &e)) { set_err(err, errlen, e); return nullptr; }
  return make(std::move(map), cfg, threads);
}
SURFSIM_API void* surfsim_create_from_memory(const uint8_t* data, int64_t size, const EnvConfig* cfg, int32_t threads,
                                             char* err, int32_t errlen) {
  auto map = std::make_shared<Map>();
  std::string e;
  if (!map->load_memory(data, static_cast<size_t>(size), &e)) { set_err(err, errlen, e); return nullptr; }
  return make(std::move(map), cfg, threads);
}
SURFSIM_API void surfsim_destroy(void* h) { delete static_cast<SimHandle*>(h); }

#define ENV(h) (static_cast<SimHandle*>(h)->env)
#define MAP(h) (*static_cast<SimHandle*>(h)->map)

SURFSIM_API int32_t surfsim_obs_dim(void* h) { return ENV(h)->obs_dim(); }
SURFSIM_API int32_t surfsim_num_envs(void* h) { return ENV(h)->num_envs(); }
SURFSIM_API int32_t surfsim_set_waypoints(void* h, const float* xyz, int32_t n) { return ENV(h)->set_waypoints(xyz, n); }
SURFSIM_API int32_t surfsim_set_spawn_pool(void* h, const PlayerState* pool, int32_t n) { return ENV(h)->set_spawn_pool(pool, n); }
SURFSIM_API void surfsim_set_teleport_fail(void* h, int32_t on) { ENV(h)->set_teleport_fail(on != 0); }
SURFSIM_API void surfsim_set_goal_box(void* h, const float* mins, const float* maxs) { ENV(h)->set_goal_box(mins, maxs); }
SURFSIM_API const uint8_t* surfsim_goal_hits(void* h) { return ENV(h)->goal_hits(); }
SURFSIM_API void surfsim_force_fail(void* h, const uint8_t* mask) { ENV(h)->force_fail(mask); }
SURFSIM_API void surfsim_reset_all(void* h, uint64_t seed, float* obs) { ENV(h)->reset_all(seed, obs); }
SURFSIM_API void surfsim_step(void* h, const int32_t* actions, float* obs, float* rewards, uint8_t* done, uint8_t* trunc,
                              float* terminal_obs) {
  ENV(h)->step(actions, obs, rewards, done, trunc, terminal_obs);
}
// Fused K-tick step; every output is a strided float row target (ptr may be null).
SURFSIM_API void surfsim_step_k(void* h, const int32_t* actions, int32_t action_stride, int32_t yaw_slot,
                                int32_t fail_slot, int32_t k, float* obs, int64_t obs_stride, float* term_obs,
                                int64_t term_obs_stride, float* rec, int64_t rec_stride, float* term_rec,
                                int64_t term_rec_stride) {
  ENV(h)->step_k(actions, action_stride, yaw_slot, fail_slot, k, RowOut{obs, obs_stride},
                 RowOut{term_obs, term_obs_stride}, RowOut{rec, rec_stride}, RowOut{term_rec, term_rec_stride});
}
SURFSIM_API void surfsim_step_k_range(void* h, int32_t lo, int32_t hi, const int32_t* actions, int32_t action_stride,
                                      int32_t yaw_slot, int32_t fail_slot, int32_t k, float* obs, int64_t obs_stride,
                                      float* term_obs, int64_t term_obs_stride, float* rec, int64_t rec_stride,
                                      float* term_rec, int64_t term_rec_stride) {
  ENV(h)->step_k_range(lo, hi, actions, action_stride, yaw_slot, fail_slot, k, RowOut{obs, obs_stride},
                       RowOut{term_obs, term_obs_stride}, RowOut{rec, rec_stride}, RowOut{term_rec, term_rec_stride});
}
// step_k_range on the pool's workers; surfsim_step_wait joins it (see EnvBatch).
SURFSIM_API void surfsim_step_k_range_async(void* h, int32_t lo, int32_t hi, const int32_t* actions,
                                            int32_t action_stride, int32_t yaw_slot, int32_t fail_slot, int32_t k,
                                            float* obs, int64_t obs_stride, float* term_obs, int64_t term_obs_stride,
                                            float* rec, int64_t rec_stride, float* term_rec, int64_t term_rec_stride) {
  ENV(h)->step_k_range_async(lo, hi, actions, action_stride, yaw_slot, fail_slot, k, RowOut{obs, obs_stride},
                             RowOut{term_obs, term_obs_stride}, RowOut{rec, rec_stride},
                             RowOut{term_rec, term_rec_stride});
}
SURFSIM_API void surfsim_step_wait(void* h) { ENV(h)->step_wait(); }
// The visiting order of the last step of [lo, hi) (offsets from lo; see EnvBatch::env_order).
SURFSIM_API void surfsim_env_order(void* h, int32_t lo, int32_t hi, int32_t* out) {
  if (lo < 0 || hi > ENV(h)->num_envs() || hi <= lo || !out) return;
  ENV(h)->env_order(lo, hi, out);
}
SURFSIM_API PlayerState* surfsim_states_ptr(void* h) { return ENV(h)->states(); }
SURFSIM_API void surfsim_get_states(void* h, PlayerState* out) {
  ENV(h)->step_wait();
  std::memcpy(out, ENV(h)->states(), sizeof(PlayerState) * static_cast<size_t>(ENV(h)->num_envs()));
}
SURFSIM_API void surfsim_set_state(void* h, int32_t env, const PlayerState* s) { ENV(h)->set_state(env, *s); }

SURFSIM_API void surfsim_trace(void* h, const float* start, const float* end, int32_t usehull, TraceOut* out) {
  Trace t;
  trace_player(MAP(h), usehull, start, end, &t);
  std::memcpy(out->endpos, t.endpos, sizeof out->endpos);
  std::memcpy(out->normal, t.normal, sizeof out->normal);
  out->dist = t.dist;
  out->fraction = t.fraction;
  out->startsolid = t.startsolid;
  out->allsolid = t.allsolid;
  out->ent = t.ent;
}
// Batched traces: n segments (float [n,6] start+end) -> fraction/endpos/normal rows.
SURFSIM_API void surfsim_trace_batch(void* h, const float* seg, int64_t n, int32_t usehull, float* out /*[n,8]*/) {
  for (int64_t i = 0; i < n; ++i) {
    Trace t;
    trace_player(MAP(h), usehull, seg + 6 * i, seg + 6 * i + 3, &t);
    float* o = out + 8 * i;
    o[0] = t.fraction;
    std::memcpy(o + 1, t.endpos, 12);
    std::memcpy(o + 4, t.normal, 12);
    o[7] = t.startsolid ? 1.f : 0.f;
  }
}
SURFSIM_API int32_t surfsim_point_contents(void* h, const float* p) { return point_contents(MAP(h), p); }
SURFSIM_API void surfsim_occupancy_grid(void* h, const float* mins, float cell, int32_t nx, int32_t ny, int32_t nz,
                                        uint8_t* out) {
  ENV(h)->occupancy_grid(mins, cell, nx, ny, nz, out);
}
SURFSIM_API void surfsim_pm_step_usercmd(void* h, PlayerState* s, float yaw, float pitch, float fmove, float smove,
                                         int32_t buttons, int32_t msec) {
  ENV(h)->pm_step_usercmd(s, yaw, pitch, fmove, smove, buttons, msec);
}
SURFSIM_API int32_t surfsim_play_step(void* h, PlayerState* s, float yaw, float pitch, float fmove, float smove,
                                      int32_t buttons, int32_t msec) {
  return ENV(h)->play_step(s, yaw, pitch, fmove, smove, buttons, msec);
}
SURFSIM_API void surfsim_pm_step_single(void* h, PlayerState* s, const int32_t* action) { ENV(h)->pm_step_single(s, action); }

SURFSIM_API int32_t surfsim_num_spawns(void* h) { return static_cast<int32_t>(MAP(h).spawns.size()); }
SURFSIM_API void surfsim_get_spawn(void* h, int32_t i, float* origin, float* yaw) {
  const Map& m = MAP(h);
  if (i < 0 || i >= static_cast<int32_t>(m.spawns.size())) { origin[0] = origin[1] = origin[2] = 0; *yaw = 0; return; }
  std::memcpy(origin, m.spawns[static_cast<size_t>(i)].origin, 12);
  *yaw = m.spawns[static_cast<size_t>(i)].yaw;
}
SURFSIM_API void surfsim_map_bounds(void* h, float* mins, float* maxs) {
  std::memcpy(mins, MAP(h).world_mins, 12);
  std::memcpy(maxs, MAP(h).world_maxs, 12);
}
// Counts: planes, hull0 nodes, clipnodes, models, solids, volumes, triggers, spawns.
SURFSIM_API void surfsim_map_counts(void* h, int32_t* out8) {
  const Map& m = MAP(h);
  out8[0] = static_cast<int32_t>(m.planes.size());
  out8[1] = static_cast<int32_t>(m.hull0.size());
  out8[2] = static_cast<int32_t>(m.clipnodes.size());
  out8[3] = static_cast<int32_t>(m.models.size());
  out8[4] = static_cast<int32_t>(m.solids.size());
  out8[5] = static_cast<int32_t>(m.volumes.size());
  out8[6] = static_cast<int32_t>(m.triggers.size());
  out8[7] = static_cast<int32_t>(m.spawns.size());
}
// Export the hull-0 tree for GPU point-contents queries: planes as float4
// (normal, dist) + int type, nodes as int3 (plane, child0, child1).
SURFSIM_API void surfsim_export_hull0(void* h, float* planes4, int32_t* ptype, int32_t* nodes3, int32_t* headnode) {
  const Map& m = MAP(h);
  for (size_t i = 0; i < m.planes.size(); ++i) {
    std::memcpy(planes4 + 4 * i, m.planes[i].normal, 12);
    planes4[4 * i + 3] = m.planes[i].dist;
    ptype[i] = m.planes[i].type;
  }
  for (size_t i = 0; i < m.hull0.size(); ++i) {
    nodes3[3 * i] = m.hull0[i].plane;
    nodes3[3 * i + 1] = m.hull0[i].child[0];
    nodes3[3 * i + 2] = m.hull0[i].child[1];
  }
  *headnode = m.models[0].headnode[0];
}
// Triangle mesh of the solid geometry (world + solid brush entities):
// float32 xyz vertices and int32 triangle indices. n_out = {vertices,
// triangles}; buffers are filled only when their capacity suffices (call
// once with zero capacities for the sizes).
SURFSIM_API int32_t surfsim_export_mesh(void* h, float* verts, int32_t cap_verts, int32_t* tris, int32_t cap_tris,
                                        int32_t* n_out) {
  const Map& m = MAP(h);
  std::vector<float> v;
  std::vector<int32_t> t;
  const float zero[3] = {0.0f, 0.0f, 0.0f};
  solid_mesh(m, 0, zero, 1.0f, v, t);
  for (const BrushEntity& s : m.solids) solid_mesh(m, s.model, s.origin, 1.0f, v, t);
  n_out[0] = static_cast<int32_t>(v.size() / 3);
  n_out[1] = static_cast<int32_t>(t.size() / 3);
  if (verts && cap_verts >= n_out[0]) std::memcpy(verts, v.data(), v.size() * sizeof(float));
  if (tris && cap_tris >= n_out[1]) std::memcpy(tris, t.data(), t.size() * sizeof(int32_t));
  return 0;
}
// Solid brush entities for GPU occupancy: per entity 10 floats = hull-0 head
// node (int32 bits), origin xyz, absmin xyz, absmax xyz. Returns the count.
SURFSIM_API int32_t surfsim_solid_entities(void* h, float* out10, int32_t cap) {
  const Map& m = MAP(h);
  int32_t n = static_cast<int32_t>(m.solids.size());
  for (int32_t i = 0; i < n && i < cap; ++i) {
    const BrushEntity& s = m.solids[static_cast<size_t>(i)];
    int32_t head = m.models[static_cast<size_t>(s.model)].headnode[0];
    std::memcpy(out10 + 10 * i, &head, 4);
    std::memcpy(out10 + 10 * i + 1, s.origin, 12);
    std::memcpy(out10 + 10 * i + 4, s.absmin, 12);
    std::memcpy(out10 + 10 * i + 7, s.absmax, 12);
  }
  return n;
}
// Trigger list: kind, model, has_dest, and bounds (for kill-zone masking).
SURFSIM_API int32_t surfsim_triggers(void* h, int32_t* kinds, float* bounds6, float* damage, int32_t cap) {
  const Map& m = MAP(h);
  int32_t n = static_cast<int32_t>(m.triggers.size());
  for (int32_t i = 0; i < n && i < cap; ++i) {
    const Trigger& t = m.triggers[static_cast<size_t>(i)];
    kinds[3 * i] = static_cast<int32_t>(t.kind);
    kinds[3 * i + 1] = t.model;
    kinds[3 * i + 2] = t.has_dest ? 1 : 0;
    std::memcpy(bounds6 + 6 * i, t.absmin, 12);
    std::memcpy(bounds6 + 6 * i + 3, t.absmax, 12);
    damage[i] = t.damage;
  }
  return n;
}
// Hull-1 containment of points in a trigger (the env's own kill test).
SURFSIM_API void surfsim_trigger_contains(void* h, int32_t trig, const float* pts, int64_t n, int32_t usehull,
                                          uint8_t* out) {
  const Map& m = MAP(h);
  const Trigger& t = m.triggers[static_cast<size_t>(trig)];
  for (int64_t i = 0; i < n; ++i) out[i] = trigger_contains(m, t, usehull, pts + 3 * i) ? 1 : 0;
}

// ---- procedural map compiler ---------------------------------------------
// brushes: float records [model, contents, nplanes, (nx, ny, nz, d) * nplanes]...
SURFSIM_API int64_t surfsim_compile_bsp(const float* brushes, int64_t nfloats, const char* entities, uint8_t* out,
                                        int64_t cap, char* err, int32_t errlen) {
  BspWriter w;
  int64_t i = 0;
  while (i < nfloats) {
    Brush b;
    b.model = static_cast<int>(brushes[i]);
    b.contents = static_cast<int>(brushes[i + 1]);
    int np = static_cast<int>(brushes[i + 2]);
    i += 3;
    for (int p = 0; p < np; ++p, i += 4) {
      BrushPlane bp{{brushes[i], brushes[i + 1], brushes[i + 2]}, brushes[i + 3]};
      b.planes.push_back(bp);
    }
    w.add_brush(b);
  }
  w.set_entities(entities ? entities : "");
  std::vector<uint8_t> img;
  std::string e;
  if (!w.build(&img, &e)) { set_err(err, errlen, e); return -1; }
  if (out && static_cast<int64_t>(img.size()) <= cap) std::memcpy(out, img.data(), img.size());
  return static_cast<int64_t>(img.size());
}

// The env batch's per-env rule set with host pointers (EnvCore bytes) — what a
// GPU env (libsurf_env.so, same process) copies to the device. Returns
// sizeof(EnvCore); copies only when cap is large enough.
SURFSIM_API int32_t surfsim_core_bytes(void* h, void* out, int32_t cap) {
  const EnvCore& c = ENV(h)->core();
  const int32_t n = static_cast<int32_t>(sizeof(EnvCore));
  if (out && cap >= n) std::memcpy(out, &c, sizeof(EnvCore));
  return n;
}
