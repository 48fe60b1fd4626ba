"""Route an installed quartz package's int8 kernels to the B200 kernels.

quartz calls its int8 path through module-level names: the kernels package
(quartz/kernels/__init__.py:10-12), its int8 and fused modules
(quartz/kernels/int8.py, quartz/kernels/fused.py), and quartz/quantize.py,
which binds ``matmul_int8``, ``warmup``, ``fused_mlp_decode`` and
``warmup_fused`` by name at import (quartz/quantize.py:20-21) -- so those
bindings are replaced too. After ``install()``, QuantizedLinear,
QuantizedEmbedding.as_linear and FusedMLP run on the GPU with their numpy
signatures unchanged.
"""

from __future__ import annotations

import importlib
from dataclasses import dataclass, field

from . import kernels as _k

# (module, attribute) -> replacement
_TARGETS = {
    "quartz.kernels.int8": {
        "w8a32_gemv": _k.w8a32_gemv,
        "w8a32_gemv_serial": _k.w8a32_gemv_serial,
        "w8a32_gemm": _k.w8a32_gemm,
        "matmul_int8": _k.matmul_int8,
        "warmup": _k.warmup,
    },
    "quartz.kernels.fused": {
        "fused_mlp_decode": _k.fused_mlp_decode,
        "warmup_fused": _k.warmup_fused,
    },
    "quartz.kernels": {
        "w8a32_gemv": _k.w8a32_gemv,
        "w8a32_gemm": _k.w8a32_gemm,
        "matmul_int8": _k.matmul_int8,
        "warmup": _k.warmup,
    },
    "quartz.quantize": {
        "matmul_int8": _k.matmul_int8,
        "warmup": _k.warmup,
        "fused_mlp_decode": _k.fused_mlp_decode,
        "warmup_fused": _k.warmup_fused,
    },
}


@dataclass
class Installation:
    """What install() replaced; uninstall() puts the originals back."""

    saved: list = field(default_factory=list)   # (module, name, original)

    def uninstall(self) -> None:
        for mod, name, orig in reversed(self.saved):
            setattr(mod, name, orig)
        self.saved.clear()


def install(modules: dict | None = None, strict: bool = True) -> Installation:
    """Patch quartz's kernel entry points in place.

    modules: optional {dotted name: module object}; names not given are
    imported. strict: raise if a target module or attribute is missing
    (otherwise skip it).
    """
    inst = Installation()
    for modname, repl in _TARGETS.items():
        mod = (modules or {}).get(modname)
        if mod is None:
            try:
                mod = importlib.import_module(modname)
            except ImportError:
                if strict:
                    inst.uninstall()
                    raise
                continue
        for name, fn in repl.items():
            if not hasattr(mod, name):
                if strict:
                    inst.uninstall()
                    raise AttributeError(f"{modname} has no attribute {name!r}")
                continue
            inst.saved.append((mod, name, getattr(mod, name)))
            setattr(mod, name, fn)
    return inst
