"""B200 (sm_100a) weight-only quantized GEMV for decode and verify widths (M <= 16).

Operators (host mirrors of the reference's kernels/sglang operator modules, computed by
the hand-written CUDA library ``_fnx.so``):

* ``w8a16_gemv``, ``bf16_gemv``, ``w8a16_gemv_silu_mul`` -- W8A16 (int8 / fp8) GEMV,
  the lm_head and draft-head path, with fused greedy argmax;
  ``w8a16_gemv_norm_gated`` -- the same GEMV with a gated RMSNorm on its input;
* ``w4a16_nvfp4_gemv`` -- NVFP4 GEMV; ``quantize_nvfp4`` / ``dequantize_nvfp4`` codec;
* ``draft_moe_gemv`` / ``moe_gemv`` -- routed NVFP4 MoE expert GEMVs (gate_up + SiLU,
  down + router-weighted route sum), M <= 16;
* ``router_gemv``, ``route_softmax_fast``, ``router_topk`` -- the MoE router projection
  and its softmax top-k routing table (fused into one launch by ``router_topk``);
* ``draft_topk1_postprocess``, ``draft_head_topk1`` -- the greedy draft step with the
  hot-vocabulary token map (the latter fused into the draft head's argmax);
* ``nvfp4_dense`` -- the NVFP4 dense lm_head: load-time packing with an on-disk cache
  and the linear method serving it through the NVFP4 GEMV;
* ``sharded`` -- vocab-sharded lm_head and expert-sharded MoE over torch.distributed;
* ``check_device_errors`` -- reads (and clears) the error flags that the kernels' bounded
  waits set when they run out of time.
"""

from .w8a16_gemv import (  # noqa: F401
    GemvConfig,
    bf16_gemv,
    dense_path,
    prealloc,
    scratch_slot,
    set_dense_path,
    w8a16_gemv,
    w8a16_gemv_norm_gated,
    w8a16_gemv_norm_gated_supported,
    w8a16_gemv_silu_mul,
    w8a16_gemv_silu_mul_supported,
)
from .w4a16_nvfp4_gemv import (  # noqa: F401
    dequantize_nvfp4,
    quantize_nvfp4,
    swizzle_blockscale,
    w4a16_nvfp4_gemv,
)
from .draft_moe_gemv import (  # noqa: F401
    DEFAULT_CONFIG,
    DraftMoeGemvConfig,
    DraftMoeGemvRunner,
    SharedExpert,
    draft_moe_gemv,
    enable_draft_moe_gemv,
    make_workspace,
    fused_tiling,
    moe_gemv,
    moe_kernel_name,
    moe_launches_per_call,
    moe_path,
    moe_plan,
    set_moe_path,
    unsupported_reason,
)

from .errors import DeviceWaitError, check_device_errors  # noqa: F401
from .router import covered, route_softmax_fast, router_gemv, router_topk  # noqa: F401
from .draft_topk1 import draft_head_topk1, draft_topk1_postprocess  # noqa: F401

__version__ = "0.1.0"
