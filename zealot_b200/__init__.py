"""zealot_b200: B200-native (sm_100a) backend for zealot-rl's PPO update.

The compute lives in ``libzealot_rl.so`` (CUDA kernels behind a C ABI,
declared in ``include/zealot_rl.h``).  ``zealot_b200.zealot_rl`` mirrors the
zealot-rl Rust API (ActorCritic, PpoConfig, PpoStats, gae, Lcg) on top of
that library; ``zealot_b200.synth`` generates seeded synthetic rollouts.
Importing this package does not load the CUDA library; the first call that
needs it does, and fails loudly if it is missing.
"""

__all__ = ["synth", "zealot_rl", "native"]
