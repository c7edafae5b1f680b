"""Route the reference package's hot-path imports to semblend_b200.

``install()`` registers this package's modules under the reference's module
names, so unchanged callers — the vLLM connector and model-runner hooks, the
TRT-LLM backend, the pipeline — import the B200 kernels:

==========================================  ====================================
reference module                            replaced by
==========================================  ====================================
``semblend_core.rope_correction``           :mod:`semblend_b200.rope_correction`
``semblend_core.triton_kernels``            :mod:`semblend_b200.triton_kernels`
``semblend_core.donor_store``               :mod:`semblend_b200.donor_store`
``semblend_core.partial_attention``         :mod:`semblend_b200.partial_attention`
``synapse_kv_connector.<same four>``        the same modules (the reference's
                                            re-export shims)
``synapse_kv_connector.cagra_donor_store``  :mod:`semblend_b200.cagra_donor_store`
==========================================  ====================================

``patch_sglang()`` additionally points the SGLang integration's
``_SemBlendDonorStore`` at :class:`semblend_b200.radix_store.RadixDonorStore`.

Call it before the first import of those names (for example at the top of the
serving entry point).  The parent packages (``semblend_core``,
``synapse_kv_connector``) are imported normally when installed, so everything
outside the hot path keeps coming from the reference.
"""

from __future__ import annotations

import importlib
import sys
import types

HOT_PATH = ("rope_correction", "triton_kernels", "donor_store", "partial_attention")
PARENTS = ("semblend_core", "synapse_kv_connector")
EXTRA = {"synapse_kv_connector.cagra_donor_store": "semblend_b200.cagra_donor_store"}


def install(parents: tuple[str, ...] = PARENTS) -> dict[str, str]:
    """Alias the hot-path modules; returns {reference name: our module name}."""
    done = {}
    for parent in parents:
        if parent not in sys.modules:
            try:
                importlib.import_module(parent)
            except ImportError:
                # no reference install: a bare package so `import parent.name` resolves
                pkg = types.ModuleType(parent)
                pkg.__path__ = []
                sys.modules[parent] = pkg
    for name in HOT_PATH:
        ours = importlib.import_module(f"semblend_b200.{name}")
        for parent in parents:
            full = f"{parent}.{name}"
            sys.modules[full] = ours
            pkg = sys.modules.get(parent)
            if pkg is not None:
                setattr(pkg, name, ours)
            done[full] = ours.__name__
    for full, ours_name in EXTRA.items():
        parent, name = full.rsplit(".", 1)
        if parent not in parents:
            continue
        ours = importlib.import_module(ours_name)
        sys.modules[full] = ours
        pkg = sys.modules.get(parent)
        if pkg is not None:
            setattr(pkg, name, ours)
        done[full] = ours.__name__
    return done


def patch_sglang() -> bool:
    """Point semblend.integration.sglang.radix_backend._SemBlendDonorStore at
    the GPU store; False if that module is not importable."""
    try:
        rb = importlib.import_module("semblend.integration.sglang.radix_backend")
    except ImportError:
        return False
    from .radix_store import RadixDonorStore, _DonorEntry

    rb._SemBlendDonorStore = RadixDonorStore
    rb._DonorEntry = _DonorEntry
    return True


def uninstall(parents: tuple[str, ...] = PARENTS) -> None:
    """Drop the aliases (the next import reloads the reference modules)."""
    names = [f"{p}.{n}" for n in HOT_PATH for p in parents] + [f for f in EXTRA if f.rsplit(".", 1)[0] in parents]
    for full in names:
        parent, name = full.rsplit(".", 1)
        mod = sys.modules.get(full)
        if mod is not None and mod.__name__.startswith("semblend_b200."):
            del sys.modules[full]
            pkg = sys.modules.get(parent)
            if pkg is not None and getattr(pkg, name, None) is mod:
                delattr(pkg, name)
