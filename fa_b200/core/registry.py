"""Backend discovery and driver lookup (mirror of the reference core/registry.py).

A backend is a module ``fa_b200/backends/<dir>/backend.py`` with a
module-level ``META`` (``fa_b200.core.contract.Meta``).  Backends are keyed
by directory name; ``META.type`` selects the driver.  Importing a backend
module stays cheap (CUDA work happens inside its functions), so discovery
runs on hosts without a GPU.

Same functions and error behaviour as the reference (registry.py:26-88):
``prepare_call``, ``discover``, ``get``, ``all_names``, ``require_attention``,
``name_of``, ``get_reference`` (exactly one reference, else ``ValueError``),
``driver_for`` (``KeyError`` for an unknown type), ``needs_compile``.
"""

import importlib
import os

_BACKENDS = None  # dirname -> module
_DRIVERS = {
    "external": "fa_b200.core.drivers.external",
}
_PACKAGE = "fa_b200.backends"


def _backends_dir():
    return os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "backends")


def prepare_call(spec, case):
    """Let an early-loading driver prepare before canonical inputs exist."""
    driver = driver_for(spec.META)
    prepare = getattr(driver, "prepare", None)
    if prepare is not None:
        return prepare(spec, case)

    def bind(canonical):
        return driver.make_call(spec, case, canonical)

    return bind


def discover(force=False):
    global _BACKENDS
    if _BACKENDS is None or force:
        found = {}
        root = _backends_dir()
        for entry in sorted(os.listdir(root)):
            if os.path.isfile(os.path.join(root, entry, "backend.py")):
                found[entry] = importlib.import_module(f"{_PACKAGE}.{entry}.backend")
        _BACKENDS = found
    return _BACKENDS


def get(name):
    return discover()[name]


def all_names(include_diagnostics=False):
    return [n for n, m in discover().items() if include_diagnostics or not m.META.diagnostic]


def require_attention(spec):
    if spec.META.diagnostic:
        raise ValueError(f"{name_of(spec)} is diagnostic-only, not an attention backend")


def name_of(spec):
    """Registry key of a backend module (independent of the legacy META.name)."""
    matches = [n for n, m in discover().items() if m is spec]
    if len(matches) != 1:
        raise ValueError(f"expected one registered name for {spec!r}, found {matches!r}")
    return matches[0]


def get_reference():
    """(name, module) of the single is_reference backend."""
    refs = [(n, m) for n, m in discover().items() if m.META.is_reference]
    if len(refs) != 1:
        raise ValueError(f"expected exactly one reference backend, found {len(refs)}")
    return refs[0]


def driver_for(meta):
    return importlib.import_module(_DRIVERS[meta.type])


def needs_compile(spec):
    driver = driver_for(spec.META)
    predicate = getattr(driver, "needs_compile", None)
    if predicate is not None:
        return bool(predicate(spec))
    return bool(getattr(driver, "requires_compile", False))
