"""Failure detection on the host: heartbeats through the rendezvous store, and the device-side
wait timeouts surfaced as Python exceptions.

A rank that dies or stops between steps must not leave the others spinning in a kernel or a
collective. Two mechanisms, neither of which needs a GPU fault to test:

  Heartbeat   every rank stores (step, wall time) under its key in the job's store after each
              step; before launching the next step a rank checks every peer's entry and raises
              PeerFailure naming the rank that is missing or stale, so nothing is launched
              that would wait for it. (Process groups are also created with a short timeout,
              which ends a collective that a dead peer never joins with an error.)
  check_device_errors
              every bounded wait inside our kernels (mbarrier waits, peer flag barriers)
              records a code in a device word when it gives up; this reads the words and
              raises DeviceWaitTimeout with the phase and peer.
"""
from __future__ import annotations

import time


class PeerFailure(RuntimeError):
    def __init__(self, rank, reason):
        super().__init__(f"rank {rank}: {reason}")
        self.rank = rank


class DeviceWaitTimeout(RuntimeError):
    pass


class Heartbeat:
    def __init__(self, store, rank: int, world: int, prefix: str = "llmt/heartbeat"):
        self.store, self.rank, self.world, self.prefix = store, rank, world, prefix

    def _key(self, r):
        return f"{self.prefix}/{r}"

    def beat(self, step: int):
        self.store.set(self._key(self.rank), f"{step}:{time.time():.3f}")

    def check(self, max_age_s: float, min_step: int | None = None):
        """Raise PeerFailure if a peer has no heartbeat, or an older one than max_age_s seconds,
        or (with min_step) has not reached that step."""
        now = time.time()
        for r in range(self.world):
            if r == self.rank:
                continue
            key = self._key(r)
            if not self.store.check([key]):
                raise PeerFailure(r, "no heartbeat")
            step, t = self.store.get(key).decode().split(":")
            if now - float(t) > max_age_s:
                raise PeerFailure(r, f"last heartbeat {now - float(t):.1f} s ago (step {step})")
            if min_step is not None and int(step) < min_step:
                raise PeerFailure(r, f"at step {step}, expected {min_step}")


def _phase(kind, code):
    if kind == "dp" or kind == "tp":
        base = (code // 100) * 100
        names = {100: "data-parallel barrier before the update", 200: "data-parallel barrier after the update",
                 300: "tensor-parallel all-gather barrier", 400: "tensor-parallel reduce-scatter barrier",
                 500: "tensor-parallel GEMM reduce-scatter barrier", 600: "tensor-parallel backward all-gather barrier",
                 700: "overlapped data-parallel bucket barrier", 800: "overlapped data-parallel final barrier"}
        return f"{names.get(base, f'barrier {base}')}, waiting for peer {code - base}"
    return f"code {code}"


def check_device_errors(reset: bool = True):
    """Raise DeviceWaitTimeout if any bounded device-side wait gave up since the last check."""
    from llmt.ops import native as N
    C = N.ext()
    codes = {"gemm": N.gemm_error_code(reset), "attention": N.attn_error_code(reset), "dp": C.dp_error_code(reset)}
    bad = {k: v for k, v in codes.items() if v}
    if bad:
        msg = "; ".join(f"{k}: {_phase(k, v)}" for k, v in bad.items())
        raise DeviceWaitTimeout(f"a device-side wait timed out ({msg})")
    return codes
