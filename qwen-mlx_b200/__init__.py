"""qwen-mlx_b200: B200-native (sm_100a) continuously batched GatedDeltaNet layer step.

The compute lives in libgdn_b200.so (C ABI: include/gdn.h).  This package
holds its build recipe (build.py), the ctypes binding (abi.py), host-side
mirrors of the reference interfaces (gdn.py for the GDN layer, hybrid.py for
the attention and MoE layers of the hybrid decoder), the scheduler binding
(sched.py), the checkpoint loader (loader.py) and the seeded synthetic data
generator shared by tests and benchmarks (synth.py).
"""
from .synth import GdnConfig, QWEN35_35B_A3B  # noqa: F401

__all__ = ["GdnConfig", "QWEN35_35B_A3B"]
