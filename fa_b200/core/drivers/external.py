"""Generic Python-callable driver (mirror of the reference core/drivers/external.py).

``build(case)`` is optional, must be CPU-safe and idempotent, and runs both
in the CPU compile phase and again right before a call is made.
``adapt(case, canonical)`` turns the canonical tensors into an opaque
argument object once; ``call(op_args)`` runs one forward and returns the
canonical output.  Nothing here depends on the backend's implementation
language: the B200 backends bind a C ABI library, the reference backend is
plain PyTorch.
"""

requires_compile = False


def needs_compile(spec):
    return callable(getattr(spec, "build", None))


def compile(spec, case):
    hook = getattr(spec, "build", None)
    if hook is None:
        return
    if not callable(hook):
        raise TypeError("external build must be callable")
    hook(case)


def make_call(spec, case, canonical):
    compile(spec, case)
    op_args = spec.adapt(case, canonical)

    def call():
        return spec.call(op_args)

    return call
