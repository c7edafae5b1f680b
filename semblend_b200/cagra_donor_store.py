"""Drop-in for synapse_kv_connector/cagra_donor_store.py: the exact GPU search
in place of cuVS CAGRA.

The reference's CAGRADonorStore keeps a host list of embeddings and rebuilds a
cuVS brute-force or CAGRA (approximate) index lazily after adds
(cagra_donor_store.py:52-207); ``make_donor_store`` picks it or the numpy
DonorStore (:354-388).  Here both names give the device-mirrored
:class:`~semblend_b200.donor_store.DonorStore`: rows are written to the device
matrix as donors arrive (no index rebuild) and every search is exact, so the
results are those of the reference's brute-force path at any size.
"""

from __future__ import annotations

import logging
import os

from .donor_store import DonorStore

logger = logging.getLogger(__name__)


def _has_cuvs() -> bool:
    """The GPU search here needs no cuVS; kept for callers that probe it."""
    return True


class CAGRADonorStore(DonorStore):
    """CAGRADonorStore's constructor (cagra_donor_store.py:68-95) over the exact
    device search; ``rebuild_every`` is accepted and has nothing to do."""

    def __init__(self, max_entries: int = 100_000, embedding_dim: int = 384, min_similarity: float = 0.60,
                 rebuild_every: int = 0, **kwargs) -> None:
        super().__init__(max_entries=max_entries, embedding_dim=embedding_dim, min_similarity=min_similarity,
                         **kwargs)
        self._rebuild_every = rebuild_every


def make_donor_store(max_entries: int = 10_000, embedding_dim: int = 384, min_similarity: float = 0.60,
                     use_cagra: bool | None = None, **kwargs) -> DonorStore:
    """make_donor_store (cagra_donor_store.py:354-388): ``use_cagra`` (or
    ``SEMBLEND_USE_CAGRA``) selects the CAGRA-named class; both are the exact
    device search."""
    if use_cagra is None:
        use_cagra = os.environ.get("SEMBLEND_USE_CAGRA", "0").lower() in ("1", "true", "yes")
    cls = CAGRADonorStore if use_cagra else DonorStore
    return cls(max_entries=max_entries, embedding_dim=embedding_dim, min_similarity=min_similarity, **kwargs)


__all__ = ["CAGRADonorStore", "make_donor_store"]
