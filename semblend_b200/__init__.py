"""semblend_b200 — B200-native (sm_100a) donor-reuse hot path for SemBlend.

Drop-in replacements for the reference's hot-path modules:

* :mod:`semblend_b200.rope_correction`  ↔ ``semblend_core.rope_correction``
* :mod:`semblend_b200.triton_kernels`   ↔ ``semblend_core.triton_kernels``
* :mod:`semblend_b200.partial_attention` ↔ ``semblend_core.partial_attention``
* :mod:`semblend_b200.donor_store`      ↔ ``semblend_core.donor_store``

:func:`semblend_b200.compat.install` aliases the reference module names (and
the ``synapse_kv_connector`` re-export shims) to these modules so unchanged
callers pick them up.  All compute runs in ``_native/libsemblend_b200.so``
(build with ``python -m semblend_b200.build``).
"""

from ._lib import NativeLibraryError, skipped_pairs

__version__ = "0.1.0"

__all__ = ["NativeLibraryError", "skipped_pairs", "__version__"]
