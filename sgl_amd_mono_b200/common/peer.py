"""Exchange regions for the in-kernel TP all-reduces (the role of the reference's
``common/peer.py:114-156`` PeerBuffer and ``common/guard.py`` error words).

Every rank allocates one region through the C-ABI (``dsv41_peer_alloc``: device memory,
zeroed, with a CUDA IPC handle), the handles are exchanged over the process group, and every
rank maps the others' (``dsv41_peer_open``). ``table`` is then a device int64 array of the tp
regions as mapped in this process, which K2 and ``dsv41_allreduce`` take. Construction is
collective and all ranks refuse together: a failure on any rank raises ``PeerMemoryError``
on every rank, after each has released what it made.

Device-side failures (a wait past its deadline, a peer's failure flag, the fault-injection
hook) land in the region's guard words; ``check()`` reads them and raises ``DeviceGuardError``.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

import torch
import torch.distributed as dist

from . import ext

IPC_HANDLE_BYTES = 64
MAX_TP = 8
GUARD_WORDS = 8
W_SEQ, W_DONE, W_DEADLINE, W_PEER, W_FAULT = 0, 1, 3, 4, 5
SITES = {1: "attention all-reduce", 2: "MoE all-reduce"}
# every exchange a wait can give up in (the fault-injection hook takes SITES only)
WAIT_SITES = {**SITES, 3: "row attention's query exchange", 4: "row attention's output exchange"}
MIN_DEADLINE_S = 0.05


class PeerMemoryError(RuntimeError):
    """The peer handshake failed on this or another rank."""


class DeviceGuardError(RuntimeError):
    """A device-side guard fired: a wait ran past its deadline, saw another rank's failure,
    or this rank's fault-injection hook skipped a push."""


class Native:
    """The C-ABI's region calls, one Python method each (tests substitute a fake)."""

    def _fn(self, name, res, args):
        f = getattr(ext.lib(), name)
        f.restype, f.argtypes = res, args
        return f

    def region_bytes(self, tp: int, cap: int) -> int:
        f = self._fn("dsv41_peer_region_bytes", ctypes.c_int64, [ctypes.c_int64, ctypes.c_int64])
        return ext.check(int(f(tp, cap)), "dsv41_peer_region_bytes")

    def alloc(self, nbytes: int) -> tuple[int, bytes]:
        f = self._fn("dsv41_peer_alloc", ctypes.c_int,
                     [ctypes.c_int64, ctypes.POINTER(ctypes.c_int64), ctypes.c_char_p])
        p = ctypes.c_int64(0)
        h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        ext.check(f(nbytes, ctypes.byref(p), h), "dsv41_peer_alloc")
        return p.value, h.raw

    def open(self, handle: bytes) -> int:
        f = self._fn("dsv41_peer_open", ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)])
        p = ctypes.c_int64(0)
        ext.check(f(handle, ctypes.byref(p)), "dsv41_peer_open")
        return p.value

    def close(self, region: int) -> None:
        ext.check(self._fn("dsv41_peer_close", ctypes.c_int, [ctypes.c_int64])(region), "dsv41_peer_close")

    def free(self, region: int) -> None:
        ext.check(self._fn("dsv41_peer_free", ctypes.c_int, [ctypes.c_int64])(region), "dsv41_peer_free")

    def status(self, region: int) -> tuple[int, list[int]]:
        f = self._fn("dsv41_peer_status", ctypes.c_int, [ctypes.c_int64, ctypes.POINTER(ctypes.c_int32)])
        words = (ctypes.c_int32 * GUARD_WORDS)()
        rc = f(region, words)
        if rc not in (0, -4):
            ext.check(rc, "dsv41_peer_status")
        return rc, list(words)


def guard_message(words: list[int]) -> Optional[str]:
    """The failure the guard words record, or None."""
    parts = []
    if words[W_DEADLINE]:
        parts.append(f"a wait at the {WAIT_SITES.get(words[W_DEADLINE], words[W_DEADLINE])} ran past its deadline")
    if words[W_PEER]:
        parts.append("a wait saw another rank's failure flag")
    if words[W_FAULT]:
        parts.append("the fault-injection hook skipped this rank's push")
    return "; ".join(parts) or None


def fault_injection(rank: int) -> Optional[tuple[int, int]]:
    """(site, after) from ``SGLANG_AMD_MONO_FAULT_INJECT`` = ``rank:site[:after]`` when it names
    this rank (the reference's test hook, ``guard.py:76-100``): the K2 launch numbered
    ``after`` (0-based) on this rank skips its push at ``site``, so the peers' waits run out."""
    spec = os.environ.get("SGLANG_AMD_MONO_FAULT_INJECT", "")
    if not spec:
        return None
    parts = spec.split(":")
    if len(parts) not in (2, 3) or not all(p.strip().isdigit() for p in parts):
        raise ValueError(f"SGLANG_AMD_MONO_FAULT_INJECT={spec!r}: want rank:site[:after]")
    r, site = int(parts[0]), int(parts[1])
    after = int(parts[2]) if len(parts) == 3 else 0
    if site not in SITES:
        raise ValueError(f"SGLANG_AMD_MONO_FAULT_INJECT site {site} not in {sorted(SITES)}")
    return (site, after) if r == rank else None


class PeerBuffer:
    """This rank's exchange region and the table of every rank's. ``cap``: bf16 elements a
    data slot holds (at least rows x hidden of the widest launch)."""

    def __init__(self, cap: int, group, rank: int, npes: int, device, native=None):
        if not 1 < npes <= MAX_TP or not 0 <= rank < npes:
            raise PeerMemoryError(f"rank {rank} of {npes}: TP 2..{MAX_TP}")
        self.native = native or Native()
        self.cap, self.rank, self.npes, self.group = -(-cap // 8) * 8, rank, npes, group
        self.local = 0
        self._opened: list[int] = []
        ok, handle, why = True, b"", ""
        try:
            self.nbytes = self.native.region_bytes(npes, self.cap)
            self.local, handle = self.native.alloc(self.nbytes)
        except Exception as e:  # noqa: BLE001 -- reported to every rank below
            ok, why = False, f"{type(e).__name__}: {e}"
        got = [None] * npes
        dist.all_gather_object(got, (ok, handle, why), group=group)
        bad = [(r, w) for r, (o, _, w) in enumerate(got) if not o]
        if bad:
            self._release()
            raise PeerMemoryError("peer region allocation failed on " +
                                  ", ".join(f"rank {r} ({w})" for r, w in bad))
        bases, ok, why = [0] * npes, True, ""
        try:
            for r, (_, h, _) in enumerate(got):
                if r == rank:
                    bases[r] = self.local
                else:
                    bases[r] = self.native.open(h)
                    self._opened.append(bases[r])
        except Exception as e:  # noqa: BLE001
            ok, why = False, f"{type(e).__name__}: {e}"
        opened = [None] * npes
        dist.all_gather_object(opened, (ok, why), group=group)
        bad = [(r, w) for r, (o, w) in enumerate(opened) if not o]
        if bad:
            self._release()
            raise PeerMemoryError("opening the peers' regions failed on " +
                                  ", ".join(f"rank {r} ({w})" for r, w in bad))
        self.bases = bases
        self.table = torch.tensor(bases, dtype=torch.int64, device=device)

    def _release(self) -> None:
        for p in self._opened:
            try:
                self.native.close(p)
            except Exception:  # noqa: BLE001 -- best effort while unwinding
                pass
        self._opened = []
        if self.local:
            try:
                self.native.free(self.local)
            except Exception:  # noqa: BLE001
                pass
            self.local = 0

    def words(self) -> list[int]:
        return self.native.status(self.local)[1]

    def check(self) -> None:
        """Raise ``DeviceGuardError`` if this rank's guard words record a failure."""
        rc, words = self.native.status(self.local)
        msg = guard_message(words)
        if rc != 0 or msg:
            raise DeviceGuardError(f"rank {self.rank}: {msg or 'device guard fired'}")

    def close(self) -> None:
        """Unmap the peers' regions and free this rank's. Collective: this rank's queued work
        is finished first (a device synchronize), then every rank meets at a barrier, so no
        rank frees its region while another rank's last exchange may still push into it or
        poll its flags."""
        if torch.cuda.is_available() and torch.cuda.is_initialized():
            torch.cuda.synchronize()
        if dist.is_available() and dist.is_initialized():
            dist.barrier(group=self.group)
        self._release()
