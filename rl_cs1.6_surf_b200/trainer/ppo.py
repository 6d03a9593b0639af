"""GPU-resident PPO trainer (reference: python/train_fast.py main loop).

Per iteration: a rollout of T decisions x K physics ticks for every env, GAE,
then E epochs x M minibatches of clipped-PPO updates. On a CUDA device:

* the simulator steps on CPU threads and writes one record row per env into
  a pinned host buffer; one async copy ships it to the GPU;
* each decision t replays a captured CUDA graph: copy in, reward of decision
  t-1 (reward kernel), depth render straight into the rollout buffer slot,
  proprio features, policy forward on the tcgen05 kernels, fused sampling,
  and the async copy of the action rows back to pinned memory;
* truncated episodes get gamma * V(s_T) from an eager render + forward of
  their terminal poses (added by the next reward kernel);
* the update replays one captured graph per epoch: permutation (keyed
  Feistel), per-minibatch advantage moments, then per minibatch the row
  gathers, forward, fused PPO loss/gradient, explicit backward, gradient
  synchronisation across ranks (data parallel) and fused clip + Adam.

On CPU the same components run through their PyTorch/numpy oracles (the
eyeless configuration trains on CPU).
"""
from __future__ import annotations

import json
import math
import os
import time
from pathlib import Path
from typing import Optional

import numpy as np
import torch

from ..models.policy import (HeadLayout, NetConfig, PolicyNet, Workspace, backward_gpu, forward_gpu,
                             space_to_depth_config)
from ..ops import rl as R
from ..rewards.spec import CpuReward, GpuReward, RewardSpec
from ..sim import mapgen
from ..sim.core import REC_COLS, STATE_DTYPE, TERM_COLS, SimCore, default_config
from ..utils.timer import PhaseClock
from .config import TrainConfig

# column layout of the per-env host record (float32)
C_OBS, C_TOBS, C_REC, C_TREC, H_COLS = 0, 16, 32, 48, 64
NOGPS = (0, 1, 2, 3, 4, 5, 6, 9, 10, 11)      # honest proprioception (no heading, no position)
REWARD_SLOT = 12                               # observation slot that carries the obs-reward feed


def build_spawn_pool(core, kind: str, cfg, procedural=None):
    """The start-state pool of a spawn mode (reference --spawn, python/train_fast.py:1391-1426):
    pool (the procedural map's drop pool, else a drop scan) | drop | platform | mixed | ramp | map."""
    from ..sim import spawns
    drops = lambda: spawns.drop_pool(core, h_range=(cfg.drop_min, cfg.drop_max),
                                     speed_range=(cfg.punch_min, cfg.punch_max), seed=cfg.map_seed + 17)
    if kind == "pool":
        return procedural if procedural is not None else drops()
    if kind == "drop":
        return drops()
    if kind == "platform":
        return spawns.platform_pool(core)
    if kind == "mixed":
        return spawns.mixed_pool(spawns.platform_pool(core), drops(), cfg.drop_frac)
    if kind == "ramp":
        return spawns.ramp_pool(core)
    if kind == "map":
        return None
    raise ValueError(f"unknown spawn mode {kind!r}")


class ReplicaDivergence(RuntimeError):
    """Data-parallel parameter replicas no longer agree."""


class Trainer:
    def __init__(self, cfg: TrainConfig, rank: int = 0, world: int = 1, comm=None, verbose: bool = True):
        cfg.validate()
        self.cfg = cfg
        self.rank, self.world, self.comm = rank, world, comm
        self.verbose = verbose and rank == 0
        self.device = torch.device(cfg.device)
        self.gpu = self.device.type == "cuda"
        torch.manual_seed(cfg.seed + 1000 * rank)
        self._setup_env()
        self._setup_net()
        self._setup_buffers()
        self.global_step = 0
        self.iteration = 0
        self._env_ready = False
        self.timer = PhaseClock(cfg.timing, self.gpu)
        self.last_stats: dict = {}

    # ---- setup ------------------------------------------------------------------------
    def _log(self, msg: str) -> None:
        if self.verbose:
            print(msg, flush=True)

    def _setup_env(self) -> None:
        cfg = self.cfg
        if cfg.map in mapgen.MAP_KINDS:
            self.procmap = mapgen.generate(cfg.map, cfg.map_seed)
            image = self.procmap.image
            self.zones = self.procmap.zones
            pool = self.procmap.spawn_pool
        else:
            self.procmap = None
            from ..sim.zones import load_zones
            image = Path(cfg.map).read_bytes()
            self.zones = load_zones(cfg.map)
            pool = None
            zp = Path(cfg.map).with_suffix(".spawns.npy")
            if zp.exists():                                   # a procedural map saved to disk keeps its pool
                pool = np.load(zp)
        self.map_image = image
        probe = None
        if cfg.spawn not in ("pool", "map") or (cfg.spawn == "pool" and pool is None):
            probe = SimCore.from_bytes(image, default_config(1), threads=1)
            pool = build_spawn_pool(probe, cfg.spawn, cfg, procedural=pool)
            probe.close()
        fixed = cfg.fix_pitch is not None
        if (cfg.respawn_frac > 0 or fixed) and pool is None:   # the reservoir / a fixed gaze need pool spawning
            from ..sim import spawns
            probe = SimCore.from_bytes(image, default_config(1), threads=1)
            pool = spawns.map_pool(probe)
            probe.close()
        if fixed:
            # fixed gaze (reference --fix-pitch, python/train_fast.py:1320-1323,
            # 1394): every start looks at the fixed pitch and the view pitch
            # rate is zero, so the pitch head cannot move the view
            pool = pool.copy()
            pool["pitch"] = np.float32(cfg.fix_pitch)
        spawn_mode = 2 if (cfg.spawn != "map" or cfg.respawn_frac > 0 or fixed) and pool is not None else 0
        env_cfg = default_config(cfg.envs, max_episode_ticks=cfg.ep_ticks, spawn_mode=spawn_mode,
                                 yaw_jitter_deg=cfg.yaw_jitter, sv_maxvelocity=cfg.maxvel,
                                 sv_airaccelerate=cfg.airaccelerate,
                                 pitch_rate_max_deg=0.0 if fixed else cfg.pitch_rate,
                                 yaw_adaptive=int(cfg.yaw_adaptive))
        self.core = SimCore.from_bytes(image, env_cfg, threads=cfg.threads)
        if spawn_mode == 2:
            self.core.set_spawn_pool(pool)
        self.spawn_pool = pool
        self.core.set_teleport_fail(cfg.teleport_fail)
        end = self.zones.get("end") if self.zones else None
        if end:
            self.core.set_goal_box(end["mins"], end["maxs"])
        self.genv = None
        if cfg.env_device == "cuda":
            if not self.gpu:
                raise ValueError("env_device cuda needs the GPU trainer (device cuda)")
            if cfg.respawn_frac > 0:
                raise ValueError("the respawn reservoir snapshots host env states: use env_device cpu with it")
            from ..sim.gpu_env import GpuEnv
            self.genv = GpuEnv(self.core, self.device)
        elif cfg.env_device != "cpu":
            raise ValueError(f"env_device must be cpu or cuda, got {cfg.env_device!r}")
        self.bounds = self.core.map_bounds()
        self.field = None
        self.field_bake_ms = None          # host-timed goal-field bake (occupancy + geodesic), race only
        self.d0 = None
        if cfg.reward.mode == "race":
            from ..ops.geodesic import bake_goal_field, euclid_goal_field
            from ..ops.vision import grid_dims
            gcell = max(cfg.lidar_cell, 16.0)
            if cfg.race_dist == "euclid":
                mn, mx = self.core.map_bounds()
                gmins, gx, gy, gz = grid_dims(mn, mx, gcell)
                self.field = euclid_goal_field(end, gmins, gcell, (gx, gy, gz), device=self.device)
            else:
                t_bake = time.perf_counter()
                self.field = bake_goal_field(self.core, end, cell=gcell, device=self.device if self.gpu else "cpu",
                                             kill_aware=cfg.race_kill_aware)
                if self.gpu:
                    torch.cuda.synchronize(self.device)
                self.field_bake_ms = 1e3 * (time.perf_counter() - t_bake)
            start = pool["origin"] if pool is not None else np.array([s[0] for s in self.core.spawns()])
            d_start = self.field.sample(start)
            ok = d_start < self.field.valid_max
            if ok.mean() < 0.5:
                raise RuntimeError("race: most start states cannot reach the finish through the goal graph"
                                   + (" (kill volumes masked as walls disconnect them)" if cfg.race_kill_aware
                                      else ""))
            self.d0 = float(np.median(d_start[ok]))
            self._log(f"goal field: reach_max {self.field.reach_max:.0f}u, start distance {self.d0:.0f}u")

    def _setup_net(self) -> None:
        cfg = self.cfg
        heads = tuple(h for h in cfg.heads if not (cfg.continuous_yaw and h == "yaw"))
        if not cfg.vision:
            heads = tuple(h for h in heads if h != "pitch")
        self.layout = HeadLayout(heads, cfg.continuous_yaw)
        self.feat_idx = tuple(range(15)) if cfg.gps else NOGPS
        self.rew_col = -1
        if cfg.obs_reward:                     # the previous reward rides in slot 12 (hidden heading / position)
            self.feat_idx = tuple(sorted(set(self.feat_idx) | {REWARD_SLOT}))
            self.rew_col = self.feat_idx.index(REWARD_SLOT)
        self.frame_ch = 2 if (cfg.vision and cfg.surf_mask) else 1
        self.n_frames = max(1, int(cfg.frame_stack)) if cfg.vision else 1
        if cfg.vision and (cfg.surf_mask or self.n_frames > 1) and not self.gpu:
            raise RuntimeError("the surface mask and frame stacking need a CUDA device")
        ncfg = NetConfig(vision=cfg.vision, img_h=cfg.lidar_h, img_w=cfg.lidar_w,
                         img_c=self.frame_ch * self.n_frames, n_scalar=len(self.feat_idx),
                         scalar_pad=16, fc=cfg.fc, proprio=cfg.proprio, hidden=cfg.hidden, mlp=tuple(cfg.mlp),
                         heads=self.layout)
        self.s2d = bool(cfg.vision and cfg.vision_s2d and self.gpu)
        if self.s2d:
            ncfg = space_to_depth_config(ncfg)
        self.net = PolicyNet(ncfg, self.device, seed=cfg.seed)
        if self.comm is not None:
            self.comm.broadcast_params(self.net)
        self.opt = R.Adam(self.net, lr=cfg.lr, eps=1e-5, max_norm=cfg.max_grad_norm)
        self.heads = R.HeadArgs(self.layout, self.device)
        if cfg.vision:
            from ..ops.vision import DepthCamera, SdfVolume
            if self.procmap is not None and "grid_mins" in self.procmap.meta:
                m = self.procmap.meta
                self.volume = SdfVolume.build(self.core, cell=m["cell"], mins=np.array(m["grid_mins"]),
                                              dims=tuple(m["dims"]), device=self.device)
            else:
                self.volume = SdfVolume.build(self.core, cell=cfg.lidar_cell, device=self.device)
            self.surf_nz = None
            if cfg.surf_mask:
                from ..ops import surfmask
                self.surf_nz, lin = surfmask.for_volume(self.core, self.volume)
                h = surfmask.histogram(lin.cpu().numpy())
                self._log(f"surface mask: {h['surfaced']:,} surfaced voxels ({h['surfable']:,} surfable, "
                          f"{h['walkable'] + h['flat']:,} walkable)")
                del lin
            from ..ops.vision import LAYOUT_NHW, LAYOUT_S2D4
            self.camera = DepthCamera(self.volume, cfg.lidar_w, cfg.lidar_h, range_units=cfg.lidar_range,
                                      near_range=cfg.lidar_near, max_steps=cfg.march_steps, pinhole=cfg.pinhole,
                                      dtype=torch.bfloat16, surf_nz=self.surf_nz,
                                      layout=LAYOUT_S2D4 if self.s2d else LAYOUT_NHW)
        self._log(f"policy: {self.net.n_params:,} parameters, heads {self.layout.heads}"
                  f"{' + continuous yaw' if self.layout.continuous_yaw else ''}")

    def _setup_buffers(self) -> None:
        cfg, dev = self.cfg, self.device
        N, T = cfg.envs, cfg.n_steps
        self.N, self.T, self.K = N, T, cfg.act_every
        self.frame = cfg.lidar_w * cfg.lidar_h * self.frame_ch if cfg.vision else 0
        self.stacker = None
        if cfg.vision and self.n_frames > 1:
            from ..ops.framestack import FrameStacker
            self.stacker = FrameStacker(self.n_frames, self.frame, self.frame_ch)
            if self.stacker.pro > T:
                raise ValueError(f"frame_stack {self.n_frames} reaches {self.stacker.pro} decisions back: "
                                 f"n_steps must be at least that")
        # decision t's frame lives in slot pro + t; slots [0, pro) hold the
        # previous rollout's last frames (the stack's reach-back)
        self.pro = self.stacker.pro if self.stacker is not None else 0
        self.img_w = self.frame * self.n_frames
        pin = self.gpu
        self.hrec = torch.zeros((N, H_COLS), dtype=torch.float32, pin_memory=pin)
        self.act_pin = torch.zeros((N, 8), dtype=torch.int32, pin_memory=pin)
        self.hdev = torch.zeros((N, H_COLS), dtype=torch.float32, device=dev)
        bf = torch.bfloat16 if self.gpu else torch.float32
        self.b_img = torch.zeros((self.pro + T + 1, N, max(self.frame, 8)), dtype=bf, device=dev) \
            if cfg.vision else None
        if self.stacker is not None:
            self.b_age = torch.zeros((T + 1, N), dtype=torch.int32, device=dev)
            self.age_cur = torch.zeros(N, dtype=torch.int32, device=dev)
        self.b_scal = torch.zeros((T + 1, N, 16), dtype=bf, device=dev)
        self.b_act = torch.zeros((T, N, 8), dtype=torch.int32, device=dev)
        self.b_logp = torch.zeros((T, N), device=dev)
        self.b_val = torch.zeros((T, N), device=dev)
        self.b_rew = torch.zeros((T, N), device=dev)
        self.b_done = torch.zeros((T, N), device=dev)
        self.adv = torch.zeros((T, N), device=dev)
        self.ret = torch.zeros((T, N), device=dev)
        self.last_val = torch.zeros(N, device=dev)
        self.moments = torch.zeros(2, dtype=torch.float64, device=dev)
        self.feat_idx_t = torch.tensor(list(self.feat_idx) + [0] * (16 - len(self.feat_idx)), dtype=torch.int32,
                                       device=dev)
        self.mb = T * N // cfg.minibatches
        self.ez = None
        if cfg.ez_eps > 0:
            self.ez = R.EzGreedy(N, cfg.ez_eps, cfg.ez_mu, cfg.ez_max, device=dev)
            self.b_ez = torch.zeros((T, N), dtype=torch.uint8, device=dev)
        # the update samples from a pool of rollout rows when it strides over
        # decisions or leaves ez-greedy bursts out (else: every row)
        self.pooled = cfg.train_stride > 1 or self.ez is not None
        self.zero_rew = torch.zeros(N, device=dev)
        if self.gpu:
            G = cfg.env_groups if (cfg.env_groups > 1 and N % cfg.env_groups == 0 and N // cfg.env_groups >= 64) else 1
            step = N // G
            self.groups = [(g * step, (g + 1) * step) for g in range(G)]
            # the order each group's depth images are rendered in: the host
            # env's spatial visiting order of the group (neighbouring cameras
            # share cached SDF bricks), identity until the first step
            self.order_pin = torch.cat([torch.arange(hi - lo, dtype=torch.int32) for lo, hi in self.groups])
            self.order_pin = self.order_pin.pin_memory()
            self.order_dev = self.order_pin.to(dev)
            self.ws_grp = [Workspace(self.net, step) for _ in range(G)]
            if self.genv is not None:
                if self.stacker is not None:
                    raise ValueError("frame stacking steps its reach-back on the host bootstrap: use env_device cpu")
                self.boot_cap = min(step, 64)
                self.ws_boot = Workspace(self.net, self.boot_cap)
                self.boot_scal = torch.zeros((self.boot_cap, 16), dtype=torch.bfloat16, device=dev)
                self.boot_img = torch.zeros((self.boot_cap, max(self.frame, 8)), dtype=torch.bfloat16, device=dev) \
                    if cfg.vision else None
                self.boot_overflow = torch.zeros((), dtype=torch.int64, device=dev)
            self.stk_grp = [torch.zeros((step, self.img_w), dtype=torch.bfloat16, device=dev) for _ in range(G)] \
                if self.stacker is not None else None
            self.grp_events = [torch.cuda.Event() for _ in range(G)]
            self._host_bound = False          # set after each host-env rollout (picks the loop)
            self.ws_upd = Workspace(self.net, self.mb)
            self.perm = torch.zeros(T * N, dtype=torch.int64, device=dev)
            if self.pooled:
                self.pool = torch.zeros(T * N, dtype=torch.int64, device=dev)
                self.pool_count = torch.zeros(1, dtype=torch.int64, device=dev)
                self.mb_graphs: list = []
            self.perm_key = torch.tensor([cfg.seed * 7919 + self.rank], dtype=torch.int64, device=dev)
            self.mom_mb = torch.zeros((cfg.minibatches, 2), dtype=torch.float64, device=dev)
            self.img_mb = torch.zeros((self.mb, max(self.img_w, 8)), dtype=torch.bfloat16, device=dev)
            self.scal_mb = torch.zeros((self.mb, 16), dtype=torch.bfloat16, device=dev)
            self.coef = torch.tensor([cfg.clip, cfg.vf, cfg.ent], dtype=torch.float32, device=dev)
            self.loss_stats = torch.zeros(6, dtype=torch.float32, device=dev)
            self.sample_counter = torch.zeros(1, dtype=torch.int64, device=dev)
            self.reward = GpuReward(cfg.reward, N, self.K, self.bounds, dev, self.field, self.d0)
            if self.comm is not None and hasattr(self.comm, "attach"):
                self.comm.attach(self.net, self.opt, self.reward)
            self.rew_graphs: list = []
            self.upd_graph = None
        else:
            self.reward = CpuReward(cfg.reward, N, self.K, self.bounds, self.field, self.d0)
        self.seed_base = (self.cfg.seed * 1_000_003 + self.rank * 7_777_777) & 0xFFFFFFFFFFFF
        self.rnd = None
        if cfg.rnd_coef > 0:
            from .rnd import RND
            self.rnd = RND(15, device=dev, seed=cfg.seed)
            self.rnd_obs = torch.zeros((T + 1, N, 15), device=dev)
        self.respawn = None
        if cfg.respawn_frac > 0:
            from .respawn import RespawnReservoir
            binned = cfg.respawn_binned > 0 and self.field is not None
            self.respawn = RespawnReservoir(
                N, cfg.respawn_reservoir, margin_ticks=int(round(cfg.respawn_margin * 100)), map_id=self._map_id(),
                seed=cfg.seed * 31 + 23, dist_fn=self.field.sample if binned else None,
                dist_max=self.d0 if binned else None, dist_valid_max=self.field.valid_max if binned else None,
                bins=max(cfg.respawn_binned, 1), rank=self.rank)
            self.start_pool = self.spawn_pool

    def _map_id(self) -> str:
        import hashlib
        return hashlib.sha1(self.map_image).hexdigest()[:16]

    def _observe_respawn(self, t: int) -> None:
        if self.respawn is None:
            return
        h = self.hrec.numpy()
        ended = (h[:, C_REC + 11] != 0) | (h[:, C_REC + 12] != 0)
        self.respawn.observe(self.core.states_view, ended, ticks=self.K, step_index=t)

    def _train_rnd(self, steps: int = 4, batch: int = 4096) -> None:
        """A few predictor updates on random observations of this rollout."""
        T, N = self.T, self.N
        if self.gpu:
            obs = self.rnd_obs[1:].reshape(-1, 15)
        else:
            obs = torch.from_numpy(self.hrec.numpy()[:, C_OBS:C_OBS + 15].copy())
        g = torch.Generator(device=obs.device).manual_seed(self.cfg.seed * 977 + self.iteration)
        for _ in range(steps):
            idx = torch.randint(0, obs.shape[0], (min(batch, obs.shape[0]),), device=obs.device, generator=g)
            self.rnd.train_step(obs[idx])
        del T, N

    def _refresh_respawn_pool(self) -> None:
        if self.respawn is None:
            return
        self.respawn.commit(self.comm if self.world > 1 else None)
        pool = self.respawn.build_pool(self.start_pool, pool_size=self.cfg.respawn_pool,
                                       fresh_frac=1.0 - self.cfg.respawn_frac,
                                       vel_scale=tuple(self.cfg.respawn_speed),
                                       pitch_jitter=0.0 if self.cfg.fix_pitch is not None else 5.0)
        self.core.set_spawn_pool(pool)

    # ---- environment plumbing -------------------------------------------------------------
    def _env_step(self) -> None:
        h = self.hrec
        base, stride = h.data_ptr(), H_COLS
        self.core.step_k(self.act_pin.data_ptr(), 8, self.K, yaw_slot=6 if self.layout.continuous_yaw else -1,
                         fail_slot=7, obs=(base + 4 * C_OBS, stride), term_obs=(base + 4 * C_TOBS, stride),
                         rec=(base + 4 * C_REC, stride), term_rec=(base + 4 * C_TREC, stride))

    def reset(self) -> None:
        """Reset every env and write the spawn records (first decision)."""
        seed = self.cfg.seed * 1009 + self.rank * 100_003
        if self.genv is not None:
            self.hdev.zero_()
            self.genv.reset(seed, obs=self.hdev[:, C_OBS:C_OBS + 15], rec=self.hdev[:, C_REC:C_REC + REC_COLS])
            self.reward.init(self.hdev[:, C_REC:C_REC + REC_COLS])
            if self.stacker is not None:
                self.age_cur.zero_()
            return
        obs = self.core.reset(seed)
        st = self.core.states_view
        h = self.hrec.numpy()
        h[:] = 0
        h[:, C_OBS:C_OBS + 15] = obs[:, :15]
        h[:, C_REC:C_REC + 3] = st["origin"]
        h[:, C_REC + 3] = st["yaw"]
        h[:, C_REC + 4] = st["pitch"]
        h[:, C_REC + 5] = st["ducked"]
        h[:, C_REC + 6:C_REC + 9] = st["velocity"]
        if self.gpu:
            self.hdev.copy_(self.hrec, non_blocking=True)
            self.reward.init(self.hdev[:, C_REC:C_REC + REC_COLS])
            if self.stacker is not None:
                self.age_cur.zero_()
        else:
            self.reward.init(h[:, C_REC:C_REC + REC_COLS].copy())

    # ---- GPU rollout ------------------------------------------------------------------------
    def _features(self, obs: torch.Tensor, out: torch.Tensor, rew: Optional[torch.Tensor] = None) -> None:
        """Proprioception rows; with obs_reward, column ``rew_col`` holds
        tanh(rew / 0.1) (the previous decision's reward; zeros when ``rew``
        is None)."""
        from ..ops import _lib
        from ..ops._lib import check, ptr, stream_ptr
        extra = None
        if self.rew_col >= 0:
            extra = rew if rew is not None else self.zero_rew[:obs.shape[0]]
        check(_lib.lib("libsurf_rl.so").surf_obs_features(ptr(obs), obs.stride(0), ptr(self.feat_idx_t),
                                                          len(self.feat_idx), 16, ptr(out), out.stride(0),
                                                          obs.shape[0], ptr(extra), self.rew_col,
                                                          stream_ptr(obs.device)),
              "surf_obs_features")

    def _group_body(self, g: int, t: int, env: bool = True) -> None:
        """GPU work of env group g at decision slot t (t == T: the rollout
        tail): upload the group's host records (GPU env: step the group's envs
        unless ``env`` is False), reward of the previous decision, depth
        render + features, policy forward, then sampling and the async copy of
        the actions to pinned memory (or, at the tail, the bootstrap value)."""
        lo, hi = self.groups[g]
        T = self.T
        if self.genv is None:
            self.hdev[lo:hi].copy_(self.hrec[lo:hi], non_blocking=True)
            self.order_dev[lo:hi].copy_(self.order_pin[lo:hi], non_blocking=True)
        elif t > 0 and env:               # the env steps on the GPU with the previous decision's actions
            self._env_body(g, t)
        if t > 0:
            last = g == len(self.groups) - 1
            self.reward(self.hdev[lo:hi, C_REC:C_REC + REC_COLS], self.b_rew[t - 1, lo:hi], self.b_done[t - 1, lo:hi],
                        lo, hi, counts=len(self.groups) == 1)
            if last and len(self.groups) > 1:
                self.reward.count_all()
            if self.rnd is not None:
                self.rnd_obs[t, lo:hi].copy_(self.hdev[lo:hi, C_OBS:C_OBS + 15])
                self.b_rew[t - 1, lo:hi].add_(self.cfg.rnd_coef * self.rnd.bonus(self.rnd_obs[t, lo:hi]))
        img = None
        if self.cfg.vision:
            img = self.b_img[self.pro + t, lo:hi]
            self.camera.render(self.hdev[lo:hi, C_REC:C_REC + 6], out=img,
                               env_order=self.order_dev[lo:hi] if self.genv is None and self.cfg.render_order else None)
            if self.stacker is not None:
                done = self.b_done[t - 1, lo:hi] if t > 0 else None      # t == 0 continues the last tail
                img = self.stacker.rollout(self.b_img, self.pro + t, lo, hi, done, self.age_cur, self.b_age[t, lo:hi],
                                           self.stk_grp[g])
        self._features(self.hdev[lo:hi, C_OBS:C_OBS + 15], self.b_scal[t, lo:hi], rew=self.b_rew[(t - 1) % T, lo:hi])
        out = forward_gpu(self.net, self.ws_grp[g], self.b_scal[t, lo:hi], img)
        vc = self.layout.value_col
        if t < T:
            R.sample_heads(out, self.heads, self.net.p("log_std"), self.b_act[t, lo:hi], self.b_logp[t, lo:hi],
                           self.seed_base ^ (0x9E3779B97F4A7C15 * (g + 1) & 0xFFFFFFFFFFFF), 0,
                           value_src=out[:, vc], value_out=self.b_val[t, lo:hi], fail_src=self.reward.stall[lo:hi],
                           counter_ptr=self.sample_counter, counter_offset=t,
                           ez=self.ez.args(lo, hi, self.b_ez[t, lo:hi]) if self.ez is not None else None)
            if self.genv is None:
                self.act_pin[lo:hi].copy_(self.b_act[t, lo:hi], non_blocking=True)
        else:
            self.last_val[lo:hi].copy_(out[:, vc])
            if g == len(self.groups) - 1:
                R.bump_counter(self.sample_counter, T)

    def _capture(self) -> None:
        """One CUDA graph per (env group, decision slot), the rollout tail included."""
        T = self.T
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for g in range(len(self.groups)):          # warm-up (kernel attributes, lazy inits)
                for t in (0, 1, T):
                    self._group_body(g, t)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.sample_counter.zero_()
        from ..ops import _lib
        self.rew_graphs = []
        self.graph_launches = []
        self.env_graphs, self.env_launches = [], []
        split = self.genv is not None          # GPU env: env steps and compute as separate graphs (two streams)
        for g in range(len(self.groups)):
            row, counts = [], []
            erow, ecounts = [None], [0]
            for t in range(T + 1):
                gr = torch.cuda.CUDAGraph()
                c0 = _lib.launch_count()
                with torch.cuda.graph(gr, stream=s):
                    self._group_body(g, t, env=not split)
                counts.append(_lib.launch_count() - c0)
                row.append(gr)
                if split and t > 0:
                    ge = torch.cuda.CUDAGraph()
                    c0 = _lib.launch_count()
                    with torch.cuda.graph(ge, stream=s):
                        self._env_body(g, t)
                    ecounts.append(_lib.launch_count() - c0)
                    erow.append(ge)
            self.rew_graphs.append(row)
            self.graph_launches.append(counts)
            self.env_graphs.append(erow)
            self.env_launches.append(ecounts)
        torch.cuda.synchronize()
        self.reset()                      # the warm-up touched env-facing reward state
        self._log(f"captured {len(self.groups) * (T + 1)} rollout graphs ({len(self.groups)} env groups)")

    def _run_group(self, g: int, t: int) -> None:
        from ..ops import _lib
        with self.timer.gpu("rollout_gpu"):
            if self.cfg.graphs:
                self.rew_graphs[g][t].replay()
                _lib.add_launches(self.graph_launches[g][t])
            else:
                self._group_body(g, t)
        self.grp_events[g].record()

    def _env_step_group(self, g: int, wait: bool = True) -> None:
        lo, hi = self.groups[g]
        h = self.hrec
        base, stride = h.data_ptr(), H_COLS
        step = self.core.step_k_range if wait else self.core.step_k_range_async
        step(lo, hi, self.act_pin.data_ptr(), 8, self.K,
             yaw_slot=6 if self.layout.continuous_yaw else -1, fail_slot=7,
             obs=(base + 4 * C_OBS, stride), term_obs=(base + 4 * C_TOBS, stride),
             rec=(base + 4 * C_REC, stride), term_rec=(base + 4 * C_TREC, stride))
        self.core.env_order(lo, hi, self.order_pin.data_ptr() + 4 * lo)

    def _env_body(self, g: int, t: int) -> None:
        """GPU env: K ticks of group g's envs with decision t-1's action rows,
        writing the observation and record rows in place, then the truncation
        bootstrap. Runs on the env stream, beside the other group's compute."""
        lo, hi = self.groups[g]
        h = self.hdev
        self.genv.step_k(self.b_act[t - 1], self.K, lo, hi, yaw_slot=6 if self.layout.continuous_yaw else -1,
                         fail_slot=7, obs=h[:, C_OBS:C_OBS + 15], term_obs=h[:, C_TOBS:C_TOBS + 15],
                         rec=h[:, C_REC:C_REC + REC_COLS], term_rec=h[:, C_TREC:C_TREC + 8])
        if self.cfg.ep_ticks:
            self._bootstrap_truncations_gpu(lo, hi)

    def _bootstrap_truncations_gpu(self, lo: int, hi: int) -> None:
        """Device-side twin of _bootstrap_truncations for envs [lo, hi): up to
        boot_cap truncated envs (stable order) get gamma * V(terminal state)
        staged for the next reward kernel, with no host round trip; more in
        one decision are counted in boot_overflow (their bootstrap is 0)."""
        h = self.hdev
        trunc = h[lo:hi, C_REC + 12] != 0
        idx = torch.argsort(trunc.to(torch.int8), descending=True, stable=True)[:self.boot_cap] + lo
        valid = h[:, C_REC + 12].index_select(0, idx) != 0
        rows = h.index_select(0, idx)
        self._features(rows[:, C_TOBS:C_TOBS + 15].contiguous(), self.boot_scal)
        img = None
        if self.cfg.vision:
            img = self.camera.render(rows[:, C_TREC:C_TREC + 6].contiguous(), out=self.boot_img)
        out = forward_gpu(self.net, self.ws_boot, self.boot_scal, img, B=self.boot_cap)
        v = self.cfg.gamma * out[:, self.layout.value_col]
        cur = self.reward.boot.index_select(0, idx)
        self.reward.boot.index_copy_(0, idx, torch.where(valid, v, cur))
        self.boot_overflow.add_((trunc.sum() - self.boot_cap).clamp_(min=0))

    def _bootstrap_truncations(self, g: int, t: int) -> None:
        """gamma * V(s_T) for envs of group g whose episode was truncated this
        decision (their states are already the next episode's): render the
        terminal poses, run the value head, stage the bonus for the group's
        next reward kernel (stream-ordered before it)."""
        lo, hi = self.groups[g]
        h = self.hrec.numpy()
        trunc = lo + np.flatnonzero(h[lo:hi, C_REC + 12] != 0)
        if len(trunc) == 0:
            return
        # the indices and the group's pinned rows go up as asynchronous copies
        # (a fancy-indexed host gather would be pageable memory, which blocks
        # the host) and the truncated rows are picked on the device. hrec[lo:hi] is not
        # rewritten before this stream's next group launch has completed
        # (the env steps the group again only after that decision's actions).
        grp = torch.empty((hi - lo, self.hrec.shape[1]), dtype=self.hrec.dtype, device=self.device)
        grp.copy_(self.hrec[lo:hi], non_blocking=True)
        idx = torch.from_numpy(trunc).pin_memory().to(self.device, non_blocking=True)
        rows = grp.index_select(0, idx - lo)                                              # [M, 64]
        M = len(trunc)
        scal = torch.zeros((M, 16), dtype=torch.bfloat16, device=self.device)
        self._features(rows[:, C_TOBS:C_TOBS + 15].contiguous(), scal)
        img = None
        if self.cfg.vision:
            img = self.camera.render(rows[:, C_TREC:C_TREC + 6].contiguous())
            if self.stacker is not None:      # the terminal state is one decision past slot pro + t
                stk = torch.empty((M, self.img_w), dtype=torch.bfloat16, device=self.device)
                img = self.stacker.terminal(self.b_img, self.pro + t, idx, img, self.age_cur, stk)
        out = forward_gpu(self.net, self.ws_grp[g], scal, img, B=M)
        self.reward.boot.index_copy_(0, idx, self.cfg.gamma * out[:, self.layout.value_col])

    def rollout_gpu(self) -> None:
        """Env groups alternate with the GPU: while the host steps group g's
        envs, the GPU works on the other group's decision."""
        T, G = self.T, len(self.groups)
        tm = self.timer
        if self.cfg.graphs and not self.rew_graphs:
            self._capture()
        if self.pro:                          # carry the last frames over as the reach-back prologue
            self.b_img[:self.pro].copy_(self.b_img[T:T + self.pro])
        if self.genv is not None:
            self._rollout_device()
            return
        for g in range(G):
            self._run_group(g, 0)
        # The overlapped loop only pays when the host is the bottleneck (it
        # costs launch latency when env workers share cores with this thread
        # while the GPU is the slower side): choose it from the previous
        # rollout's split between waiting for the GPU and stepping envs.
        if G > 1 and self.cfg.async_env and self._host_bound:
            wait_s, env_s = self._rollout_host_async()
        else:
            wait_s, env_s = self._rollout_host_sync()
        self._host_bound = wait_s < 0.05 * env_s

    def _rollout_host_sync(self) -> tuple:
        """One group at a time: wait for its GPU work, step its envs (this
        thread and the workers), launch its next decision. Returns the seconds
        spent waiting for the GPU and stepping envs."""
        T, G = self.T, len(self.groups)
        tm = self.timer
        wait_s = env_s = 0.0
        for t in range(T):
            for g in range(G):
                t0 = time.perf_counter()
                with tm.phase("wait_gpu"):
                    self.grp_events[g].synchronize()
                t1 = time.perf_counter()
                with tm.phase("env"):
                    self._env_step_group(g)
                t2 = time.perf_counter()
                wait_s += t1 - t0
                env_s += t2 - t1
                if self.cfg.ep_ticks:
                    self._bootstrap_truncations(g, t)
                self._run_group(g, t + 1)
            self._observe_respawn(t)
            self.global_step += self.N * self.K * self.world
        return wait_s, env_s

    def _rollout_host_async(self) -> tuple:
        """The host-env rollout with the next group's env step started on the
        simulator's workers before this thread launches the finished group's
        GPU work (truncation bootstrap, graph replay), so those launches
        overlap env stepping instead of following it -- when the next group's
        GPU work is already done (the host is the bottleneck); otherwise the
        launches go first so the GPU stays fed, as in the synchronous loop.
        Groups own disjoint rows of the action and record buffers; the respawn
        reservoir reads every env's state, so with it on the first group of a
        decision starts after the observation."""
        T, G = self.T, len(self.groups)
        tm = self.timer
        seq = [(t, g) for t in range(T) for g in range(G)]
        started = -1                       # index in seq of the env step in flight
        wait_s = env_s = 0.0

        def start(i: int) -> None:
            nonlocal started, wait_s, env_s
            g2 = seq[i][1]
            t0 = time.perf_counter()
            with tm.phase("wait_gpu"):
                self.grp_events[g2].synchronize()
            t1 = time.perf_counter()
            self._env_step_group(g2, wait=False)
            wait_s += t1 - t0
            env_s += time.perf_counter() - t1
            started = i

        start(0)
        for i, (t, g) in enumerate(seq):
            t0 = time.perf_counter()
            with tm.phase("env"):
                self.core.step_wait()
            env_s += time.perf_counter() - t0
            last = g == G - 1
            if (i + 1 < len(seq) and not (last and self.respawn is not None)
                    and self.grp_events[seq[i + 1][1]].query()):
                start(i + 1)
            if self.cfg.ep_ticks:
                self._bootstrap_truncations(g, t)
            self._run_group(g, t + 1)
            if last:
                self._observe_respawn(t)
                self.global_step += self.N * self.K * self.world
            if i + 1 < len(seq) and started != i + 1:
                start(i + 1)
        return wait_s, env_s

    def _rollout_device(self) -> None:
        """The rollout with the env on the GPU: every step is device work, so
        the host only enqueues. Group g's env step (env stream) waits for its
        sampled actions and runs beside the other group's reward / render /
        forward (compute stream); the compute stream keeps the groups'
        decisions in order (the curiosity counts' two-phase rule)."""
        from ..ops import _lib
        T, G = self.T, len(self.groups)
        C = torch.cuda.current_stream()
        if getattr(self, "env_stream", None) is None:
            self.env_stream = torch.cuda.Stream()
            self.ev_env = [torch.cuda.Event() for _ in range(G)]
            self.ev_sample = [torch.cuda.Event() for _ in range(G)]
        E = self.env_stream
        E.wait_stream(C)
        for t in range(T + 1):
            for g in range(G):
                if t > 0:
                    E.wait_event(self.ev_sample[g])
                    with torch.cuda.stream(E):
                        if self.cfg.graphs:
                            self.env_graphs[g][t].replay()
                            _lib.add_launches(self.env_launches[g][t])
                        else:
                            self._env_body(g, t)
                    self.ev_env[g].record(E)
                    C.wait_event(self.ev_env[g])
                with self.timer.gpu("rollout_gpu"):
                    if self.cfg.graphs:
                        self.rew_graphs[g][t].replay()
                        _lib.add_launches(self.graph_launches[g][t])
                    else:
                        self._group_body(g, t, env=False)
                self.ev_sample[g].record(C)
            if t < T:
                self.global_step += self.N * self.K * self.world
        C.wait_stream(E)

    # ---- GPU update ---------------------------------------------------------------------------
    def _epoch_prologue(self) -> None:
        """The epoch's permutation of the sample rows (all rows, or the pool)
        and the per-minibatch advantage moments (reduced across ranks)."""
        from ..ops import _lib
        from ..ops._lib import check, ptr, stream_ptr
        T, N, mb, nmb = self.T, self.N, self.mb, self.cfg.minibatches
        if self.pooled:
            R.permutation_pool(self.perm, self.pool, self.pool_count, self.perm_key)
        else:
            check(_lib.lib("libsurf_rl.so").surf_permutation(ptr(self.perm), T * N, ptr(self.perm_key),
                                                             stream_ptr(self.device)), "surf_permutation")
        self.mom_mb.zero_()
        R.adv_moments(self.adv.view(-1), self.perm, mb, nmb, self.mom_mb)
        if self.comm is not None:
            self.comm.allreduce_moments(self.mom_mb)

    def _minibatch(self, m: int) -> None:
        """Minibatch m of the epoch: row gathers, forward, fused PPO loss and
        gradient, backward, optimizer step (fused across ranks)."""
        from ..ops import gemm as G
        T, N, mb = self.T, self.N, self.mb
        f_img = self.b_img[self.pro:self.pro + T].view(T * N, -1) if self.cfg.vision else None
        f_scal = self.b_scal[:T].view(T * N, 16)
        idx = self.perm[m * mb:(m + 1) * mb]
        if self.stacker is not None:
            self.stacker.gather(self.b_img, idx, self.b_age[:T].view(-1), self.img_mb)
        elif self.cfg.vision:
            G.gather_rows(f_img, idx, self.img_mb)
        G.gather_rows(f_scal, idx, self.scal_mb)
        out = forward_gpu(self.net, self.ws_upd, self.scal_mb, self.img_mb if self.cfg.vision else None)
        R.ppo_loss(out, self.layout.value_col, self.b_act.view(T * N, 8), self.b_logp.view(-1),
                   self.adv.view(-1), self.ret.view(-1), idx, self.mom_mb[m], self.heads, self.net.p("log_std"),
                   self.coef, float(mb * self.world), self.ws_upd.dout16, self.net.g("log_std"), self.loss_stats)
        hook = None
        if self.comm is not None and getattr(self.comm, "nbuckets", 0):
            # the tower / FC gradient is reduced across ranks on a side stream
            # while the convolutions' backward runs on this one
            main, side = torch.cuda.current_stream(self.device), self._side_stream()

            def hook():
                side.wait_stream(main)
                with torch.cuda.stream(side):
                    self.comm.bucket(0)
        backward_gpu(self.net, self.ws_upd, self.scal_mb, on_towers=hook)
        if hook is not None:
            torch.cuda.current_stream(self.device).wait_stream(self._side_stream())
        if self.comm is not None:
            self.comm.step(self.net, self.opt)          # fused reduce-scatter (rest) + clip + Adam + push
        else:
            self.opt.step()

    def _side_stream(self):
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(self.device)
        return self._side

    def _epoch_body(self) -> None:
        self._epoch_prologue()
        for m in range(self.cfg.minibatches):
            self._minibatch(m)

    def _snapshot(self):
        return (self.net.flat.clone(), self.opt.m.clone(), self.opt.v.clone(), self.opt.hyper.clone())

    def _restore(self, snap) -> None:
        """Undo a warm-up step so the first real update starts from the same weights."""
        self.net.flat.copy_(snap[0]); self.opt.m.copy_(snap[1]); self.opt.v.copy_(snap[2])
        self.opt.hyper.copy_(snap[3]); self.net.sync_bf16(); self.net.grad.zero_()
        self.loss_stats.zero_()

    def _pool_minibatches(self) -> int:
        """Build this iteration's sample pool and return the minibatches per
        epoch: floor(pool / mb), the same on every rank (reference: the pool
        trimmed to a multiple of the minibatch, python/train_fast.py:2162-2186)."""
        cfg = self.cfg
        offset = (self.iteration - 1) % cfg.train_stride          # rotates so no phase goes unseen
        R.train_pool(self.b_ez if self.ez is not None else None, self.T, self.N, cfg.train_stride, offset,
                     self.pool, self.pool_count)
        nmb = int(self.pool_count.item()) // self.mb                # one host read per iteration
        if self.comm is not None:
            nmb = -int(self.comm.max_scalar(-nmb))                  # every rank steps the optimizer alike
        return min(nmb, cfg.minibatches)

    def _update_pooled_gpu(self) -> None:
        from ..ops import _lib
        cfg = self.cfg
        nmb = self._pool_minibatches()
        self.last_minibatches = nmb
        if not cfg.graphs:
            for _ in range(cfg.epochs):
                self._epoch_prologue()
                for m in range(nmb):
                    self._minibatch(m)
            return
        if not self.mb_graphs:
            # one graph for the prologue and one per minibatch position: the
            # number replayed follows the pool size of the iteration
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            snap = self._snapshot()
            with torch.cuda.stream(s):
                self._epoch_prologue()
                self._minibatch(0)                              # warm-up outside capture
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            self._restore(snap)
            self.pro_graph = torch.cuda.CUDAGraph()
            c0 = _lib.launch_count()
            with torch.cuda.graph(self.pro_graph, stream=s):
                self._epoch_prologue()
            self.pro_launches = _lib.launch_count() - c0
            self.mb_launches = []
            for m in range(cfg.minibatches):
                g = torch.cuda.CUDAGraph()
                c0 = _lib.launch_count()
                with torch.cuda.graph(g, stream=s):
                    self._minibatch(m)
                self.mb_launches.append(_lib.launch_count() - c0)
                self.mb_graphs.append(g)
            torch.cuda.synchronize()
            self._log(f"captured the pooled update graphs (prologue + {cfg.minibatches} minibatches)")
        for _ in range(cfg.epochs):
            self.pro_graph.replay()
            _lib.add_launches(self.pro_launches)
            for m in range(nmb):
                self.mb_graphs[m].replay()
                _lib.add_launches(self.mb_launches[m])

    def update_gpu(self) -> None:
        from ..ops import _lib
        cfg = self.cfg
        frac = min(1.0, self.global_step / max(1.0, cfg.steps))
        ent = cfg.ent if cfg.ent_final is None else cfg.ent + (cfg.ent_final - cfg.ent) * frac
        self.coef[2] = ent
        self.moments.zero_()
        R.gae(self.b_rew, self.b_val, self.b_done, self.last_val, cfg.gamma ** self.K, cfg.gae, self.adv, self.ret,
              self.moments)
        self.loss_stats.zero_()
        if self.pooled:
            self._update_pooled_gpu()
            return
        if cfg.graphs:
            if self.upd_graph is None:
                s = torch.cuda.Stream()
                s.wait_stream(torch.cuda.current_stream())
                snap = self._snapshot()
                with torch.cuda.stream(s):
                    self._epoch_body()                         # warm-up outside capture
                torch.cuda.current_stream().wait_stream(s)
                torch.cuda.synchronize()
                self._restore(snap)
                self.upd_graph = torch.cuda.CUDAGraph()
                c0 = _lib.launch_count()
                with torch.cuda.graph(self.upd_graph, stream=s):
                    self._epoch_body()
                self.upd_launches = _lib.launch_count() - c0
                torch.cuda.synchronize()
                self._log("captured the update graph (one epoch)")
            for _ in range(cfg.epochs):
                self.upd_graph.replay()
                _lib.add_launches(self.upd_launches)
        else:
            for _ in range(cfg.epochs):
                self._epoch_body()

    # ---- CPU path -------------------------------------------------------------------------------
    def _cpu_obs(self, t: int) -> None:
        h = self.hrec.numpy()
        feats = np.zeros((self.N, 16), np.float32)
        feats[:, :len(self.feat_idx)] = h[:, [C_OBS + i for i in self.feat_idx]]
        if self.rew_col >= 0:
            feats[:, self.rew_col] = np.tanh(self.b_rew[(t - 1) % self.T].numpy() / 0.1)
        self.b_scal[t].copy_(torch.from_numpy(feats))
        if self.cfg.vision:
            raise RuntimeError("the vision policy needs a CUDA device (the depth camera is a GPU kernel)")

    def rollout_cpu(self) -> None:
        T = self.T
        gen = torch.Generator().manual_seed(self.cfg.seed * 31 + self.iteration * 1_000_003 + self.rank * 7919)
        for t in range(T):
            self._cpu_obs(t)
            with torch.no_grad():
                out = self.net.forward_reference(self.b_scal[t], None)
                act, logp = R.sample_reference(out, self.layout, self.net.p("log_std"), gen)
            if self.ez is not None:
                self.b_ez[t].copy_(self.ez.apply_reference(act, self.layout, gen))
            stall = getattr(self, "_stall", None)
            if stall is not None:
                act[:, 7] = torch.from_numpy(stall.astype(np.int32))
            self.b_act[t].copy_(act)
            self.b_logp[t].copy_(logp)
            self.b_val[t].copy_(out[:, self.layout.value_col])
            self.act_pin.copy_(act)
            self._env_step()
            self._observe_respawn(t)
            h = self.hrec.numpy()
            boot = None
            trunc = np.flatnonzero(h[:, C_REC + 12] != 0)
            if len(trunc):
                feats = np.zeros((len(trunc), 16), np.float32)
                feats[:, :len(self.feat_idx)] = h[trunc][:, [C_TOBS + i for i in self.feat_idx]]
                if self.rew_col >= 0:
                    feats[:, self.rew_col] = 0.0
                with torch.no_grad():
                    v = self.net.forward_reference(torch.from_numpy(feats), None)[:, self.layout.value_col]
                boot = np.zeros(self.N, np.float32)
                boot[trunc] = self.cfg.gamma * v.numpy()
            r, d, self._stall = self.reward(h[:, C_REC:C_REC + REC_COLS].copy(), boot)
            if self.rnd is not None:
                r = r + self.cfg.rnd_coef * self.rnd.bonus(torch.from_numpy(h[:, C_OBS:C_OBS + 15].copy())).numpy()
            self.b_rew[t].copy_(torch.from_numpy(r))
            self.b_done[t].copy_(torch.from_numpy(d))
            self.global_step += self.N * self.K * self.world
        self._cpu_obs(T)
        with torch.no_grad():
            self.last_val.copy_(self.net.forward_reference(self.b_scal[T], None)[:, self.layout.value_col])

    def update_cpu(self) -> dict:
        cfg = self.cfg
        adv, ret = R.gae_reference(self.b_rew, self.b_val, self.b_done, self.last_val, cfg.gamma ** self.K, cfg.gae)
        self.adv.copy_(adv)
        self.ret.copy_(ret)
        T, N, mb = self.T, self.N, self.mb
        frac = min(1.0, self.global_step / max(1.0, cfg.steps))
        ent = cfg.ent if cfg.ent_final is None else cfg.ent + (cfg.ent_final - cfg.ent) * frac
        stats = np.zeros(4)
        gen = torch.Generator().manual_seed(self.cfg.seed * 7919 + self.rank * 104729 + self.iteration)
        pool, nmb = None, cfg.minibatches
        if self.pooled:
            offset = (self.iteration - 1) % cfg.train_stride
            pool = R.train_pool_reference(self.b_ez if self.ez is not None else None, T, N, cfg.train_stride, offset)
            nmb = len(pool) // mb
            if self.comm is not None:
                nmb = -int(self.comm.max_scalar(-nmb))
            nmb = min(nmb, cfg.minibatches)
        self.last_minibatches = nmb
        for _ in range(cfg.epochs):
            perm = torch.randperm(T * N, generator=gen) if pool is None else pool[torch.randperm(len(pool), generator=gen)]
            for m in range(nmb):
                idx = perm[m * mb:(m + 1) * mb]
                a = self.adv.view(-1)[idx]
                moments = None
                if self.comm is not None:      # global advantage moments (sum, sum of squares, count)
                    mom = torch.stack([a.double().sum(), (a.double() ** 2).sum(), torch.tensor(float(mb)).double()])
                    self.comm.allreduce_moments(mom)
                    moments = mom
                params = self.net.autograd_params()
                out = self.net.forward_reference(self.b_scal[:T].reshape(T * N, 16)[idx], None, params)
                loss, pg, vl, en = R.ppo_loss_reference(out, self.layout.value_col, self.b_act.view(T * N, 8)[idx],
                                                        self.b_logp.view(-1)[idx], a, self.ret.view(-1)[idx],
                                                        self.layout, params["log_std"], cfg.clip, cfg.vf, ent,
                                                        moments=moments)
                (loss / self.world).backward()          # the summed gradient is the global-mean gradient
                self.net.collect_grads(params)
                if self.comm is not None:
                    self.comm.step(self.net, self.opt)
                else:
                    self.opt.step_reference()
                stats += [pg.item(), vl.item(), en.item(), 1.0]
        n = max(stats[3], 1.0)
        return {"policy_loss": stats[0] / n, "value_loss": stats[1] / n, "entropy": stats[2] / n}

    # ---- iteration ------------------------------------------------------------------------------
    def _check_replicas(self) -> None:
        """Every ``replica_check_every`` iterations, compare the ranks'
        parameter checksums (one collective pair, taken by every rank at the
        same iteration, so all ranks raise together). Reference: the parameter
        checksum of the data-parallel design, docs/ddp-plan.md:448-460."""
        every = int(getattr(self.cfg, "replica_check_every", 0) or 0)
        if self.comm is None or every <= 0 or self.iteration % every:
            return
        lo, hi = self.comm.checksum(self.net)
        if lo != hi:
            raise ReplicaDivergence(f"iteration {self.iteration}: parameter replicas differ across ranks "
                                    f"(checksum min {lo!r}, max {hi!r})")

    def train_iteration(self) -> dict:
        tm = self.timer
        tm.new_iteration()
        if not self._env_ready:              # first iteration of this process (fresh or resumed run)
            self.reset()
            self._env_ready = True
        self.iteration += 1
        self.reward.set_step(self.global_step)
        with tm.phase("rollout"):
            if self.gpu:
                self.rollout_gpu()
            else:
                self.rollout_cpu()
        if self.rnd is not None:
            with tm.phase("rnd"):
                self._train_rnd()
        with tm.phase("respawn"):
            self._refresh_respawn_pool()
        with tm.phase("update"):
            loss = self._update_and_stats()
        self._check_replicas()
        stats = dict(self.reward.pop_stats(), **loss)
        stats["global_step"] = self.global_step
        stats["iteration"] = self.iteration
        stats["timing"] = tm.collect()
        self.last_stats = stats
        return stats

    def _update_and_stats(self) -> dict:
        if self.gpu:
            with self.timer.gpu("update_gpu"):
                self.update_gpu()
            if self.comm is not None:
                self.comm.merge_counts(self.reward)
            ls = self.loss_stats.tolist()
            # kernels record bounded-wait timeouts and out-of-range indices in
            # the device error flag instead of faulting: raise here
            from ..ops.gemm import check_error_flag
            check_error_flag(self.device)
            if self.comm is not None and hasattr(self.comm, "check"):
                self.comm.check()
            n = max(ls[5], 1.0)
            loss = {"policy_loss": ls[0] / n, "value_loss": ls[1] / n, "entropy": ls[2] / n, "approx_kl": ls[3] / n,
                    "clip_frac": ls[4] / n}
        else:
            loss = self.update_cpu()
        return loss

    def release_graphs(self) -> None:
        """Drop every captured CUDA graph (graphs holding NCCL calls must be
        released before the process group is destroyed)."""
        if self.gpu:
            torch.cuda.synchronize()
            self.rew_graphs = []
            self.env_graphs = []
            self.upd_graph = None
            self.pro_graph = None
            if self.pooled:
                self.mb_graphs = []
            import gc
            gc.collect()
            torch.cuda.synchronize()

    # ---- checkpoints ----------------------------------------------------------------------------
    def state_dict(self) -> dict:
        counts = None
        if self.cfg.reward.int_coef > 0:
            c = self.reward.counts
            counts = (c.cpu().numpy() if torch.is_tensor(c) else c).astype(np.uint32)
        opt = self.opt.state_dict()
        policy = self.net.state_dict()
        if self.comm is not None and hasattr(self.comm, "full_optimizer_state"):
            opt.update({k: v.cpu() for k, v in self.comm.full_optimizer_state(self.opt).items()})
            policy["flat"] = self.comm.full_params(self.net).detach().cpu()
        return {"format": "surfb200-ckpt-1", "policy": policy, "optimizer": opt,
                "global_step": self.global_step, "iteration": self.iteration, "config": self.cfg.to_dict(),
                "int_counts": counts, "respawn": self.respawn.state_dict() if self.respawn is not None else None,
                "rnd": self.rnd.state_dict() if self.rnd is not None else None}

    def load_state_dict(self, sd: dict, reset_steps: bool = False, reset_counts: bool = False) -> None:
        self.net.load_state_dict(sd["policy"])
        self.opt.load_state_dict(sd["optimizer"])
        if not reset_steps:
            self.global_step = int(sd["global_step"])
            self.iteration = int(sd.get("iteration", 0))
        if self.rnd is not None and sd.get("rnd"):
            self.rnd.load_state_dict(sd["rnd"])
        if self.respawn is not None and sd.get("respawn"):
            if not self.respawn.load_state_dict(sd["respawn"]) and self.verbose:
                print("respawn reservoir not restored (empty, or recorded on another map)")
        c = sd.get("int_counts")
        if c is not None and not reset_counts and self.cfg.reward.int_coef > 0:
            if len(c) == len(self.reward.counts):
                src = torch.as_tensor(np.asarray(c).astype(np.int64))
                if torch.is_tensor(self.reward.counts):
                    self.reward.counts.copy_(src.to(torch.int32).to(self.reward.counts.device))
                else:
                    self.reward.counts[:] = np.asarray(c)
