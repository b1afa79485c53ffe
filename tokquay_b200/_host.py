"""The Tokquay package this library plugs into.

``tokquay_b200`` is a drop-in for Tokquay's paged path, not a second copy of
Tokquay: the reference's own ``Sequence`` / ``SamplingParams``,
``Scheduler``, ``Engine`` and its allocator bookkeeping run unchanged on top
of this package's ``BlockAllocator`` (a subclass of the reference's that only
adds the device step view) and ``GPT2`` (the fused paged forward).  So the
reference package ``tokquay`` must be importable.

When it is not on ``sys.path``, the install next to this checkout
(``<checkout>/baseline/_ref``, made by ``baseline/install_ref.sh``) is used if
present; otherwise importing this package fails with an error that says so.
"""

from __future__ import annotations

import importlib
import sys
from pathlib import Path

_CHECKOUT_INSTALL = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def _import_tokquay():
    try:
        return importlib.import_module("tokquay")
    except ImportError:
        pass
    if (_CHECKOUT_INSTALL / "tokquay" / "__init__.py").is_file():
        sys.path.append(str(_CHECKOUT_INSTALL))
        try:
            return importlib.import_module("tokquay")
        except ImportError:
            pass
    raise ImportError(
        "tokquay_b200 plugs into the Tokquay package `tokquay`, which is not importable: install it "
        "(baseline/install_ref.sh <tokquay checkout>) or put its checkout on PYTHONPATH")


tokquay = _import_tokquay()

from tokquay import engine as ref_engine  # noqa: E402
from tokquay import generate as ref_generate  # noqa: E402
from tokquay import kv_cache as ref_kv_cache  # noqa: E402
from tokquay import model as ref_model  # noqa: E402
from tokquay import scheduler as ref_scheduler  # noqa: E402
from tokquay import sequence as ref_sequence  # noqa: E402

__all__ = ["tokquay", "ref_engine", "ref_generate", "ref_kv_cache", "ref_model", "ref_scheduler", "ref_sequence"]
