"""B200-native drafter training step for the parallel_eagle drafter.

A drop-in for the reference's training path (``pe.config``, ``pe.masks``,
``pe.nn``, ``pe.drafter``, ``pe.partition``, ``pe.train``): same classes,
functions, dataclasses and checkpoint layout, with every op running in the
hand-written sm_100a kernels of ``libpe_b200.so`` (C ABI in
``include/pe_b200.h``).  There is no CPU fallback.

``install_as_pe()`` registers this package under the reference's module names
so existing ``import pe.partition`` call sites resolve here.
"""

from __future__ import annotations

import importlib
import sys

__version__ = "0.1.0"

_MODULES = ("config", "masks", "nn", "drafter", "partition", "train", "features", "target")


def install_as_pe() -> None:
    """Alias this package as ``pe`` (and ``pe.<module>``) in ``sys.modules``.

    The draft proposals live in one module here; it also answers to the
    reference's ``pe.decode``, ``pe.decode.tree``, ``pe.decode.chain`` and
    ``pe.decode.verify``."""
    sys.modules["pe"] = sys.modules[__name__]
    for m in _MODULES:
        sys.modules[f"pe.{m}"] = importlib.import_module(f"{__name__}.{m}")
    dec = importlib.import_module(f"{__name__}.decode")
    for sub in ("tree", "chain", "verify"):
        sys.modules[f"pe.decode.{sub}"] = dec
        setattr(dec, sub, dec)
    sys.modules["pe.decode"] = dec
