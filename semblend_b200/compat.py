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
==========================================  ====================================

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
    return done


def uninstall(parents: tuple[str, ...] = PARENTS) -> None:
    """Drop the aliases (the next import reloads the reference modules)."""
    for name in HOT_PATH:
        for parent in parents:
            full = f"{parent}.{name}"
            mod = sys.modules.get(full)
            if mod is not None and mod.__name__.startswith("semblend_b200."):
                del sys.modules[full]
                pkg = sys.modules.get(parent)
                if pkg is not None and getattr(pkg, name, None) is mod:
                    delattr(pkg, name)
