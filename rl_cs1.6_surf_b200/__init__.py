"""surfb200 — a Blackwell-native (B200, sm_100a) reinforcement-learning
framework for GoldSrc / Counter-Strike 1.6 surf.

Layers (bottom up):

* ``sim``       C++ movement simulator over BSP v30 clip hulls (libsurfsim.so),
                procedural BSP maps, zones, spawn pools.
* ``ops``       hand-written sm_100a CUDA kernels (SDF depth render, SDF/EDT
                bake, geodesic bake, tcgen05 GEMMs, action sampling, GAE,
                PPO loss, curiosity hash, fused Adam) behind a C ABI.
* ``models``    the policy networks (Nature CNN vision policy, eyeless MLP).
* ``rewards``   race / progress / coverage / speed rewards (GPU + CPU oracle).
* ``parallel``  data parallelism over NVLink: NCCL baseline and fused P2P
                all-reduce + clip + Adam, curiosity-count and moment merges.
* ``trainer``   GPU-resident PPO with CUDA graphs; ``cli`` is the front end.
* ``utils``     timing, logging, checkpoints, recording, respawn reservoir.
"""
__version__ = "0.1.0"
