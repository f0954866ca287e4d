"""b200_fa_fp32 -- sm_100a flash-attention forward, FP32 softmax variant.

The B200 counterpart of the reference's CCE FP32 backend
(backends/cce_fa_nk_nz_vector_fp32_v5_sumpack): FP32 row max, exp2 and row
sums; P in FP16 only as the tensor-core operand; O accumulated in FP32 in
tensor memory and normalized in FP32 before the FP16 store.

External-type backend; see backends/b200_fa_fp16/backend.py for the hook
contract.  Kernel symbol: ``b200_fa_fp32_kernel``.
"""

from fa_b200.core.contract import Meta

VARIANT = "fp32"

META = Meta(
    name="b200_fa_fp32",
    type="external",
    op_type="b200_fa_fp32_kernel",
    author="fa_b200",
    notes="tcgen05/TMEM warp-specialised FA forward; FP32 softmax, FP32 O in TMEM",
)


def build(case):
    from fa_b200 import build as nvcc_build

    nvcc_build.build()


def adapt(case, canonical):
    from fa_b200.ops import Operator

    return {"q": canonical["q"], "k": canonical["k"], "v": canonical["v"],
            "scale": case.scale, "op": Operator(VARIANT)}


def call(op_args):
    return op_args["op"](op_args["q"], op_args["k"], op_args["v"], scale=op_args["scale"])
