"""constellation_b200: B200-native (sm_100a) MoE-layer hot path of Constellation.

sigmoid group-limited top-k routing -> expert-sorted dispatch -> grouped FP8 E4M3
(128x128 block-scaled) SwiGLU experts -> fp32 weighted combine with the shared expert,
behind the reference's interfaces:

* ``constellation_b200.moe_layer_runtime`` -- the Python interface of
  ``server/moe_layer_runtime.py`` (``route_token_real``, ``run_moe_layer``,
  ``run_topk_moe_layer``, ``dispatch_topk_experts``, ``infer_one_expert``,
  ``combine_outputs_torch``), plus batched variants;
* ``constellation_b200.fp8_utils`` / ``expert_placement`` -- the helper modules of the
  same names;
* ``include/constellation_b200.h`` -- the C ABI that the reference node's
  ``BackendWorkspaceV2`` / ``BackendRegistryEntryV2`` hooks bind to.

The CUDA library is loaded lazily by the modules that need it, so the pure host
helpers import without a GPU.
"""

__all__ = ["context", "moe_layer_runtime", "fp8_utils", "expert_placement", "synthetic"]
