"""Backend metadata and the backend/driver contracts of the harness.

Mirror of the reference harness contract (core/contract.py:1-62): the same
``Meta`` record and ``KernelNameError``, the same split between *backends*
(``backends/<dir>/backend.py``: ``META`` plus hooks) and *drivers*
(``core/drivers/<type>.py``: how a backend type is built and called).  The
orchestrator and runner only ever touch ``META`` and the driver.

Backend module contract, by ``META.type``:

  "external"  optional idempotent, CPU-safe ``build(case)``;
              ``adapt(case, canonical) -> op_args`` (opaque);
              ``call(op_args) -> canonical output`` ([B,Hq,Nq,128] on the
              inputs' device).  This is the type of the B200 backends and of
              the FP32 reference backend.

The reference's "tilelang" and "ascendc" types wrap Ascend toolchains that do
not exist on a CUDA host; they are not registered here, so ``driver_for``
raises ``KeyError`` for them exactly as it does for any unknown type.

Driver module contract:
  requires_compile: bool
  needs_compile(spec) -> bool                      (optional)
  compile(spec, case) -> None
  prepare(spec, case) -> bind(canonical)           (optional)
  make_call(spec, case, canonical) -> Callable[[], Tensor]
"""

from dataclasses import dataclass


class KernelNameError(ValueError):
    """A backend broke the harness's kernel-symbol contract (fatal in bench)."""


@dataclass(frozen=True)
class Meta:
    name: str                   # legacy label; the registry keys backends by directory
    type: str                   # driver type, "external" here
    op_type: str                # fallback kernel-name filter for profiling
    is_reference: bool = False  # exactly one backend is the correctness reference
    author: str = ""
    date: str = ""
    notes: str = ""
    diagnostic: bool = False    # not an attention implementation; excluded from checks
