"""pocketlm_b200 -- PocketLM's MoE expert hot path, rebuilt for NVIDIA B200 (sm_100a).

Modules:
  native   drop-in mirror of the reference's native bridge entry points,
           backed by libmoe_b200.so (include/moe_b200.h)
  runtime  layer-level entry points (run_fp8_router / run_fp8_moe on the GPU)
  synth    seeded synthetic layers in the reference's weight formats
  build    nvcc build of libmoe_b200.so for sm_100a
"""

from . import native, runtime, synth  # noqa: F401

__all__ = ["native", "runtime", "synth"]
