"""Donor -> target position mappings, on the host and on the device.

The reference carries the pairs that drive RoPE correction as Python lists:
``PositionMapping`` (semblend_core/pipeline.py:62-80) and, for a target
stitched from several donors, ``MultiDonorPositionMapping``
(semblend_core/multi_donor_types.py:50-78), which the connector's hook turns
into a list of tuples and a tensor once per layer
(synapse_kv_connector/model_runner_hook.py:495-555).  The host classes here
keep those fields and properties so code written for them keeps working;
:class:`DevicePositionMapping` is their device form: int32 pair vectors
(plus a per-pair donor index for several donors) built once per request --
from the host lists, or straight from a device chunk alignment without a host
round trip -- and accepted by the inject and permutation entry points.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib


@dataclass
class PositionMapping:
    """Host pair lists: the KV at ``donor_positions[i]`` goes to
    ``target_positions[i]`` with K rotated by their difference
    (pipeline.py:62-80)."""

    donor_positions: list[int] = field(default_factory=list)
    target_positions: list[int] = field(default_factory=list)

    @property
    def num_pairs(self) -> int:
        return len(self.donor_positions)

    @property
    def needs_correction(self) -> bool:
        """True if some pair moves its row (a non-zero RoPE delta)."""
        return any(d != t for d, t in zip(self.donor_positions, self.target_positions))


@dataclass(frozen=True)
class MultiDonorPositionMapping:
    """Host pair lists with the donor that owns each pair
    (multi_donor_types.py:50-78)."""

    donor_ids: tuple[str, ...] = ()
    donor_positions: tuple[int, ...] = ()
    target_positions: tuple[int, ...] = ()

    @property
    def num_pairs(self) -> int:
        return len(self.target_positions)

    @property
    def needs_correction(self) -> bool:
        return any(d != t for d, t in zip(self.donor_positions, self.target_positions))

    def for_donor(self, donor_id: str) -> MultiDonorPositionMapping:
        """The pairs owned by one donor, in their original order."""
        keep = [i for i, d in enumerate(self.donor_ids) if d == donor_id]
        return MultiDonorPositionMapping(
            donor_ids=tuple(self.donor_ids[i] for i in keep),
            donor_positions=tuple(self.donor_positions[i] for i in keep),
            target_positions=tuple(self.target_positions[i] for i in keep),
        )


@dataclass
class DevicePositionMapping:
    """Position pairs in device memory.

    ``donor_positions`` / ``target_positions`` are int32 vectors of equal
    length; entries past ``n_pairs`` may be -1 padding (a chunk alignment's
    arrays), which every inject entry point skips (and counts as skipped).
    ``n_pairs`` is a Python int or a device int64 scalar.  With several donors,
    ``donor_ids`` names them and ``donor_index`` (int32, per pair) points into
    it.  Building one costs no host synchronisation; ``num_pairs``,
    ``needs_correction`` and :meth:`for_donor` read device data and synchronise.
    """

    donor_positions: torch.Tensor
    target_positions: torch.Tensor
    n_pairs: int | torch.Tensor
    donor_ids: tuple[str, ...] = ()
    donor_index: torch.Tensor | None = None

    def __post_init__(self) -> None:
        for t, name in ((self.donor_positions, "donor_positions"), (self.target_positions, "target_positions")):
            _lib.require_cuda(t, name)
            if t.ndim != 1 or t.dtype != torch.int32:
                raise TypeError(f"{name} must be a 1-D int32 device tensor")
        if self.donor_positions.shape != self.target_positions.shape:
            raise ValueError("donor_positions and target_positions differ in length")
        if self.donor_index is not None and self.donor_index.shape != self.donor_positions.shape:
            raise ValueError("donor_index must have one entry per pair")

    # -- construction ----------------------------------------------------------
    @classmethod
    def from_host(cls, mapping, device) -> DevicePositionMapping:
        """Upload a :class:`PositionMapping`, a :class:`MultiDonorPositionMapping`
        or any object with ``donor_positions`` / ``target_positions`` (and
        optionally ``donor_ids``) sequences: one pinned host buffer, one copy."""
        dpos = np.asarray(mapping.donor_positions, dtype=np.int64)
        tpos = np.asarray(mapping.target_positions, dtype=np.int64)
        if dpos.shape != tpos.shape:
            raise ValueError("donor_positions and target_positions differ in length")
        if dpos.size and (min(dpos.min(), tpos.min()) < -(2**31) or max(dpos.max(), tpos.max()) >= 2**31):
            raise ValueError("positions must fit in int32")
        ids = tuple(getattr(mapping, "donor_ids", ()) or ())
        rows = [dpos, tpos]
        names: tuple[str, ...] = ()
        if ids:
            if len(ids) != dpos.shape[0]:
                raise ValueError("donor_ids must have one entry per pair")
            names = tuple(dict.fromkeys(ids))
            lookup = {n: i for i, n in enumerate(names)}
            rows.append(np.fromiter((lookup[d] for d in ids), dtype=np.int64, count=len(ids)))
        host = torch.from_numpy(np.stack(rows).astype(np.int32))
        if torch.cuda.is_available():
            host = host.pin_memory()
        dev = host.to(torch.device(device), non_blocking=True)
        return cls(dev[0], dev[1], int(dpos.shape[0]), names, dev[2] if ids else None)

    @classmethod
    def from_alignment(cls, alignment) -> DevicePositionMapping:
        """The pairs of a device chunk alignment
        (:class:`semblend_b200.alignment.DeviceAlignment`), without reading
        its pair count back: the arrays are already -1 padded."""
        return cls(alignment.donor_positions, alignment.target_positions, alignment.n_pairs)

    # -- the reference's properties -------------------------------------------
    @property
    def device(self) -> torch.device:
        return self.donor_positions.device

    @property
    def num_pairs(self) -> int:
        return int(self.n_pairs.item()) if isinstance(self.n_pairs, torch.Tensor) else int(self.n_pairs)

    def _valid(self) -> tuple[torch.Tensor, torch.Tensor]:
        n = self.num_pairs
        return self.donor_positions[:n], self.target_positions[:n]

    @property
    def needs_correction(self) -> bool:
        d, t = self._valid()
        return bool((d != t).any().item()) if d.numel() else False

    def for_donor(self, donor_id: str) -> DevicePositionMapping:
        """The pairs owned by one donor, in their original order."""
        if self.donor_index is None:
            raise ValueError("this mapping has no per-pair donor index")
        if donor_id not in self.donor_ids:
            e = self.donor_positions[:0]
            return DevicePositionMapping(e, e.clone(), 0, (donor_id,), None)
        n = self.num_pairs
        sel = torch.nonzero(self.donor_index[:n] == self.donor_ids.index(donor_id)).flatten()
        return DevicePositionMapping(self.donor_positions[sel], self.target_positions[sel], int(sel.numel()),
                                     (donor_id,), None)

    def to_host(self):
        """The host form: :class:`PositionMapping`, or
        :class:`MultiDonorPositionMapping` when donors are named."""
        d, t = self._valid()
        d, t = d.cpu().tolist(), t.cpu().tolist()
        if self.donor_index is None:
            return PositionMapping(d, t)
        idx = self.donor_index[: len(d)].cpu().tolist()
        return MultiDonorPositionMapping(tuple(self.donor_ids[i] for i in idx), tuple(d), tuple(t))


__all__ = ["DevicePositionMapping", "MultiDonorPositionMapping", "PositionMapping"]
