"""torch_fp32_ref -- the harness's correctness reference on CUDA hosts.

Takes the role ``npu_fa`` has in the reference harness
(backends/npu_fa/backend.py: ``is_reference=True``, external type), which
wraps the closed NPU operator ``torch_npu.npu_fusion_attention`` and cannot
run here.  It computes the reference's FP32 formula ``ref_flash_attn``
(backends/expert_v2/impl_tl.py:701-717): FP32 softmax(Q K^T * scale) V with
the GQA head map kv = h / (Hq/Hkv), non-causal, on the inputs' device, with
TF32 disabled.  It returns the FP32 result (before the reference's final
FP16 cast) so the harness checks O against FP32 attention, the bar of the
B200 backends (max-abs <= 2e-3, mean-abs <= 2e-4).

Blocks of query rows keep the score matrix bounded (1024 x Nk FP32).
"""

from fa_b200.core.contract import Meta

META = Meta(
    name="torch_fp32_ref",
    type="external",
    op_type="torch_fp32_ref",
    is_reference=True,
    author="fa_b200",
    notes="FP32 PyTorch attention (ref_flash_attn semantics), reference for all checks",
)

ROWS_PER_BLOCK = 1024


def adapt(case, canonical):
    return {"q": canonical["q"], "k": canonical["k"], "v": canonical["v"], "scale": case.scale}


def call(op_args):
    import torch

    q, k, v, scale = op_args["q"], op_args["k"], op_args["v"], op_args["scale"]
    B, Hq, Nq, D = q.shape
    group = Hq // k.shape[1]
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        with torch.no_grad():
            out = torch.empty((B, Hq, Nq, D), dtype=torch.float32, device=q.device)
            for b in range(B):
                for h in range(Hq):
                    kf = k[b, h // group].float()
                    vf = v[b, h // group].float()
                    for r0 in range(0, Nq, ROWS_PER_BLOCK):
                        s = (q[b, h, r0:r0 + ROWS_PER_BLOCK].float() @ kf.T) * scale
                        out[b, h, r0:r0 + ROWS_PER_BLOCK] = torch.softmax(s, dim=-1) @ vf
            return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
