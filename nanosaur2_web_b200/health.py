"""Peer liveness for the multi-GPU paths (one process per GPU).

A rank that crashes or leaves between steps must not leave the others waiting inside an NCCL
collective: a collective that never completes holds their GPUs until the process-group timeout, and
a kernel waiting on a peer would never end.  The step gate here makes the others find out on the
host, before they enqueue the next step's collectives:

* ``StepGate.enter(step)``: each rank writes ``<prefix>/<step>/<rank>`` into the rendezvous store
  (the TCPStore torch.distributed already runs) and waits, with a deadline, until every rank's key
  for that step is there.  A missing rank raises ``PeerTimeout`` naming it; nothing was launched for
  that step, so the survivors can abort cleanly.
* ``abort_process_group()``: tears the communicators down without waiting for the missing peer
  (``ncclCommAbort`` under ProcessGroupNCCL's abort, or destroy for gloo).
* ``init_process_group_bounded(...)``: the process group with a short timeout and NCCL's
  non-blocking communicator mode, so that even a collective already in flight ends with an error
  instead of blocking forever.

The reference has no multi-device code; this is the failure-detection plan of the B200 build for its
sequence-sharded and batch-sharded paths (every C-ABI call returns a status, and every device-side
wait in the kernels is bounded).
"""

from __future__ import annotations

import datetime
import os
import time
from typing import List, Optional


class PeerTimeout(RuntimeError):
    """Raised by StepGate.enter when some ranks did not reach the step before the deadline."""

    def __init__(self, step: int, missing: List[int], timeout_s: float):
        self.step, self.missing, self.timeout_s = step, list(missing), timeout_s
        super().__init__(f"ranks {self.missing} did not reach step {step} within {timeout_s:.1f} s")


class StepGate:
    """Pre-step rendezvous of all ranks over a torch.distributed store, with a deadline."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 30.0, prefix: str = "nsa_gate"):
        if world < 1 or not 0 <= rank < world:
            raise ValueError("bad rank / world")
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = float(timeout_s), prefix

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def enter(self, step: int) -> None:
        """Announce this rank at ``step`` and return once every rank has; raise PeerTimeout with the
        ranks still missing at the deadline."""
        self.store.set(self._key(step, self.rank), "1")
        deadline = time.monotonic() + self.timeout_s
        pending = [r for r in range(self.world) if r != self.rank]
        while pending:
            pending = [r for r in pending if not self.store.check([self._key(step, r)])]
            if not pending:
                break
            if time.monotonic() >= deadline:
                raise PeerTimeout(step, pending, self.timeout_s)
            time.sleep(0.01)


def default_store():
    """The store of the default process group (the rendezvous TCPStore)."""
    import torch.distributed.distributed_c10d as c10d
    return c10d._get_default_store()


def init_process_group_bounded(backend: str, rank: int, world: int, timeout_s: float = 60.0, device=None):
    """init_process_group with a short collective timeout.  For NCCL the communicators are created in
    non-blocking mode (TORCH_NCCL_USE_COMM_NONBLOCKING=1, ncclCommInitRankConfig with blocking = 0),
    so a communicator whose peer is gone can be aborted while it is still initialising, and eagerly
    when ``device`` is given."""
    import torch.distributed as dist
    if backend == "nccl":
        os.environ.setdefault("TORCH_NCCL_USE_COMM_NONBLOCKING", "1")
    kw = {}
    if backend == "nccl" and device is not None:
        kw["device_id"] = device
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s), **kw)


def abort_process_group(group=None) -> None:
    """Tear the process group down without waiting for missing peers: ProcessGroupNCCL's abort
    (ncclCommAbort on every communicator), or destroy for other backends."""
    import torch.distributed as dist
    if not dist.is_initialized():
        return
    backend: Optional[str] = None
    try:
        backend = dist.get_backend(group)
    except Exception:
        pass
    if backend == "nccl":
        import torch.distributed.distributed_c10d as c10d
        abort = getattr(c10d, "_abort_process_group", None)
        if abort is not None:
            abort(group) if group is not None else abort()
            return
    dist.destroy_process_group(group)
