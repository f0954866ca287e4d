"""torch_sdpa -- the GPU vendor's fused attention, timed beside the B200 kernels.

Takes the comparison role of the reference harness's ``npu_fa`` backend
(backends/npu_fa/backend.py), which wraps the NPU vendor's fused operator
``torch_npu.npu_fusion_attention`` and is the "Torch" row of the reference's
published table (README.md:13-17).  On B200 the vendor's fused attention is
cuDNN's scaled-dot-product attention, reached through
``torch.nn.functional.scaled_dot_product_attention`` with only the cuDNN
backend allowed (``SDPBackend.CUDNN_ATTENTION``): FP16 in, FP16 out,
non-causal, the case's scale.

K/V are expanded to the Hq query heads (kv head = h / (Hq/Hkv)) in ``adapt``,
outside the timed call, so the timed call is the attention alone.  It is
library code, not part of this build's path and not the correctness
reference (``torch_fp32_ref`` is); the harness checks its output against the
reference like any other backend's.  It needs a CUDA device.
"""

from fa_b200.core.contract import Meta

META = Meta(
    name="torch_sdpa",
    type="external",
    op_type="torch_sdpa",
    is_reference=False,
    author="fa_b200",
    notes="cuDNN fused attention via torch SDPA (fp16, BHND, non-causal, K/V expanded to Hq heads)",
)


def adapt(case, canonical):
    k, v = canonical["k"], canonical["v"]
    group = case.heads_q // case.heads_kv
    if group > 1:
        k = k.repeat_interleave(group, dim=1)
        v = v.repeat_interleave(group, dim=1)
    return {"q": canonical["q"], "k": k.contiguous(), "v": v.contiguous(), "scale": case.scale}


def call(op_args):
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    with torch.no_grad(), sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
        return F.scaled_dot_product_attention(op_args["q"], op_args["k"], op_args["v"], scale=op_args["scale"])
