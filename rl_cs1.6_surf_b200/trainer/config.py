"""Run configuration (the self-describing part of every checkpoint).

Mirrors the reference trainer's flag set (python/train_fast.py:694-993) for
the features this framework implements; ``RUN_DEFINING`` lists the keys a
bare ``--ckpt`` resume restores from the checkpoint unless the flag is given
again on the command line (reference restore logic: train_fast.py:1009-1211).
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field, fields
from typing import Optional

from ..rewards.spec import RewardSpec

# keys restored from a checkpoint unless given on the command line
RUN_DEFINING = (
    "map", "map_seed", "ep_ticks", "n_steps", "act_every", "epochs", "minibatches", "lr", "gamma", "gae", "clip",
    "ent", "ent_final", "vf", "max_grad_norm", "spawn", "teleport_fail", "yaw_jitter", "maxvel", "airaccelerate",
    "vision", "lidar_w", "lidar_h", "lidar_range", "lidar_near", "lidar_cell", "pinhole", "march_steps",
    "vision_s2d", "surf_mask", "frame_stack",
    "continuous_yaw", "gps", "heads", "hidden", "fc", "proprio", "mlp", "reward", "pitch_rate", "yaw_adaptive",
    "respawn_frac", "respawn_margin", "respawn_reservoir", "train_stride", "drop_frac", "drop_min", "drop_max",
    "punch_min", "punch_max", "respawn_speed", "respawn_binned", "respawn_pool", "rnd_coef",
    "ez_eps", "ez_mu", "ez_max", "fix_pitch", "reward_per_decision", "obs_reward", "eval_greedy_only",
    "race_dist", "race_kill_aware",
)


@dataclass
class TrainConfig:
    # map / environment
    map: str = "field"                 # procedural kind (ramps | field | race) or a .bsp path
    map_seed: int = 0
    envs: int = 2048                   # per rank
    ep_ticks: int = 6000               # truncation (ticks)
    spawn: str = "pool"                # pool (procedural drop pool) | drop | platform | mixed | ramp | map
    drop_frac: float = 0.5             # mixed: fraction of drop starts
    drop_min: float = 400.0            # drop height above the face (units)
    drop_max: float = 800.0
    punch_min: float = 100.0           # drop horizontal speed (u/s)
    punch_max: float = 400.0
    teleport_fail: bool = True
    yaw_jitter: float = 8.0
    maxvel: float = 3500.0             # sv_maxvelocity (surf servers)
    airaccelerate: float = 100.0
    pitch_rate: float = 10.0
    yaw_adaptive: bool = False
    # fixed gaze: view pitch frozen at this angle (degrees, + up) for every
    # spawn; the pitch head stays in the action space but cannot move the view
    fix_pitch: Optional[float] = None
    # PPO
    steps: float = 1e9                 # physics ticks (all ranks)
    n_steps: int = 128                 # decisions per rollout
    act_every: int = 3                 # physics ticks per decision
    epochs: int = 4
    minibatches: int = 8
    train_stride: int = 1              # update samples decisions t = offset, offset + S, ... (offset rotates)
    # ez-greedy temporally-extended exploration (0 = off): burst start
    # probability per decision, zeta exponent and cap of the burst length
    ez_eps: float = 0.0
    ez_mu: float = 2.0
    ez_max: int = 60
    lr: float = 3e-4
    gamma: float = 0.9995              # per tick; GAE uses gamma ** act_every
    gae: float = 0.95
    clip: float = 0.2
    ent: float = 0.005
    ent_final: Optional[float] = None
    vf: float = 0.5
    max_grad_norm: float = 0.5
    # vision
    vision: bool = True
    lidar_w: int = 128
    lidar_h: int = 64
    lidar_range: float = 2000.0
    lidar_near: Optional[float] = None
    lidar_cell: float = 16.0
    pinhole: bool = False
    march_steps: int = 64
    vision_s2d: bool = True            # camera renders 4x4 space-to-depth; conv1 runs as an implicit GEMM on it
    surf_mask: bool = False            # second image channel: the hit surface's |n_z| (floor / ramp / wall)
    frame_stack: int = 0               # K > 1: current frame + the decisions 1, 2, 4, 8 back as K channels
    # network
    continuous_yaw: bool = False
    gps: bool = False
    heads: tuple = ("yaw", "pitch", "fwd", "side", "jump", "duck")
    fc: int = 512
    proprio: int = 256
    hidden: int = 512
    mlp: tuple = (256, 256)
    # reward
    reward: RewardSpec = field(default_factory=RewardSpec)
    # rewards are evaluated once per decision of act_every ticks (potential
    # terms telescope exactly; stall / finish bookkeeping has decision
    # granularity); the per-tick evaluation is not provided
    reward_per_decision: bool = True
    # race shaping distance: geodesic (baked through the free voxels) or euclid
    # (straight line to the finish box, no bake); kill-aware: fail nets are
    # walls of the geodesic goal graph
    race_dist: str = "geodesic"
    race_kill_aware: bool = False
    # the previous decision's reward, tanh(r / 0.1), as an extra observation
    # scalar (the heading slot 12 that the no-GPS policy hides); race only
    obs_reward: bool = False
    # respawn reservoir (Go-Explore restarts)
    respawn_frac: float = 0.0          # share of episodes started from the reservoir (0 = off)
    respawn_margin: float = 10.0       # seconds before an episode's end that are still harvestable
    respawn_reservoir: int = 100_000
    respawn_speed: tuple = (0.9, 1.1)  # spawn speed multiplier range of reservoir starts
    respawn_binned: int = 0            # distance bins for reservoir sampling (race; 0 = uniform)
    respawn_pool: int = 4096
    # random network distillation novelty (0 = off)
    rnd_coef: float = 0.0
    # run
    seed: int = 0
    device: str = "cuda"
    graphs: bool = True
    env_groups: int = 2                # rollout: env groups alternating host stepping with GPU work
    async_env: bool = True             # host env: start the next group's step before this group's launches
    render_order: bool = True          # host env: render each group in the env step's spatial order
    env_device: str = "cpu"            # cpu: C++ thread pool + pinned rows; cuda: the same env rules on the GPU
    comm: str = "p2p"                  # p2p (fused NVLink kernels) | nccl (library baseline)
    threads: Optional[int] = None
    run: str = "runs/default"
    ckpt_every: float = 50e6
    record_every: float = 0.0
    eval_eps: int = 3
    eval_greedy_only: bool = False     # skip the stochastic eval recording
    timing: bool = False
    # data parallel: every this many iterations all ranks compare a checksum of
    # their parameter replicas and raise ReplicaDivergence if they differ (0: off)
    replica_check_every: int = 0

    def validate(self) -> None:
        """Reject settings this build cannot honour (with the reason)."""
        if self.train_stride < 1:
            raise ValueError("train_stride must be >= 1")
        if self.ez_eps < 0 or self.ez_eps >= 1:
            raise ValueError("ez_eps must be in [0, 1)")
        if self.ez_eps > 0 and (self.ez_mu <= 1.0 or self.ez_max < 1):
            raise ValueError("ez-greedy needs ez_mu > 1 and ez_max >= 1")
        if self.ez_eps > 0 and self.continuous_yaw:
            raise ValueError("ez-greedy bursts draw discrete head categories: not available with continuous_yaw")
        if not self.reward_per_decision:
            raise ValueError("rewards are evaluated once per decision in this framework (reward_per_decision must "
                             "stay on); per-tick evaluation is not provided")
        if self.obs_reward and self.reward.mode != "race":
            raise ValueError("obs_reward needs the race reward (its observation mirrors the geodesic shaping)")
        if self.obs_reward and self.gps:
            raise ValueError("obs_reward uses scalar slot 12, which gps exposes as a position channel")
        if self.race_dist not in ("geodesic", "euclid"):
            raise ValueError("race_dist must be geodesic or euclid")
        if self.race_kill_aware and self.race_dist == "euclid":
            raise ValueError("race_kill_aware masks the geodesic goal graph; the euclid field has no graph")
        if self.fix_pitch is not None and not -70.0 <= self.fix_pitch <= 30.0:
            raise ValueError("fix_pitch must lie in the view clamp [-70, 30] degrees")

    def to_dict(self) -> dict:
        d = asdict(self)
        d["reward"] = self.reward.to_dict()
        d["heads"] = list(self.heads)
        d["mlp"] = list(self.mlp)
        d["respawn_speed"] = list(self.respawn_speed)
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "TrainConfig":
        kw = {}
        names = {f.name for f in fields(cls)}
        if "vision_s2d" not in d:
            kw["vision_s2d"] = False          # saved before the space-to-depth layout: NHW image, 8x8 conv1
        for k, v in d.items():
            if k not in names:
                continue
            if k == "reward":
                v = RewardSpec.from_dict(v)
            elif k in ("heads", "mlp", "respawn_speed"):
                v = tuple(v)
            kw[k] = v
        return cls(**kw)


def bench_config(n_envs: int = 2048) -> TrainConfig:
    """The vision-PPO benchmark configuration: 2048 envs per GPU on the
    512-brush procedural map, ramp drop spawns 400-800u with random
    velocity / yaw / gaze, 128x64 depth + proprioception, Nature-CNN policy,
    PPO gamma 0.9995 / lambda 0.95 / 4 epochs / 8 minibatches / clip 0.2,
    curiosity 0.25 keyed on position x speed x gaze."""
    return TrainConfig(
        map="field", envs=n_envs, ep_ticks=6000, n_steps=128, act_every=3, epochs=4, minibatches=8,
        gamma=0.9995, gae=0.95, clip=0.2,
        reward=RewardSpec(mode="coverage", int_coef=0.25, int_cell=256.0, int_view=8, int_speed=8))


def race_bench_config(n_envs: int = 2048) -> TrainConfig:
    """The race benchmark (8-GPU config 5, per rank): the procedural linear
    race track (40 chained ramps, 4 gap jumps over teleport fail nets, a
    finish curtain), the GPU Bellman-Ford geodesic bake over the free voxels
    at 16u, potential shaping on the geodesic distance to the finish with a
    15 s stall kill, and the benchmark's network, PPO settings and curiosity."""
    return TrainConfig(
        map="race", envs=n_envs, ep_ticks=6000, spawn="pool", n_steps=128, act_every=3, epochs=4, minibatches=8,
        gamma=0.9995, gae=0.95, clip=0.2, lidar_cell=16.0,
        reward=RewardSpec(mode="race", int_coef=0.25, int_cell=256.0, int_view=8, int_speed=8, stall_secs=15.0))
