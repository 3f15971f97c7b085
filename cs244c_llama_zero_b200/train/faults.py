"""Host-side fault injection for failure-detection tests.

Faults are made on the host only - a rank that exits, raises or stops joining between steps - so
failure handling can be exercised without faulting, trapping or hanging a GPU.  The injected rank
has no kernel or collective of its own in flight when it leaves; the other ranks learn of it from
their next collective (gloo: connection closed; NCCL: the process-group timeout) and the launcher
(torchrun) tears the job down with a non-zero exit code, which the experiment harness records.

``ZB_FAULT`` holds comma-separated directives, each ``<kind>:<rank>@<step>``:

* ``kill_rank:R@S``  - rank R leaves with ``os._exit(ZB_FAULT_EXIT_CODE)`` (default 43) at the start of step S,
* ``raise_rank:R@S`` - rank R raises :class:`FaultInjected` at the start of step S,
* ``stall_rank:R@S`` - rank R stops joining: it sleeps ``ZB_FAULT_STALL_S`` seconds (default 3600) at the
  start of step S, so the others' process-group timeout (``--pg-timeout-s``) ends their next collective.
* ``skip_signal:R@S`` - rank R omits (does not launch) its next NVLink collective kernel after the start of
  step S, so it never posts that kernel's barrier signal.  The other ranks' barrier waits expire after
  ``ZB_COMM_TIMEOUT_S``, their kernels record the expiry and return, and the host raises
  ``CommTimeoutError`` at its next error check.  Needs ``--collective-impl nvls|p2p``.
"""

from __future__ import annotations

import os
import sys
import time
from dataclasses import dataclass
from typing import List, Optional

KINDS = ("kill_rank", "raise_rank", "stall_rank", "skip_signal")


class FaultInjected(RuntimeError):
    """Raised by a ``raise_rank`` directive."""


@dataclass(frozen=True)
class Fault:
    kind: str
    rank: int
    step: int


def parse_faults(spec: Optional[str]) -> List[Fault]:
    out = []
    for item in (spec or "").split(","):
        item = item.strip()
        if not item:
            continue
        try:
            kind, rest = item.split(":", 1)
            rank, step = rest.split("@", 1)
            fault = Fault(kind.strip(), int(rank), int(step))
        except ValueError as exc:
            raise ValueError(f"bad ZB_FAULT directive {item!r}; expected <kind>:<rank>@<step>") from exc
        if fault.kind not in KINDS:
            raise ValueError(f"unknown ZB_FAULT kind {fault.kind!r}; expected one of {KINDS}")
        out.append(fault)
    return out


class FaultInjector:
    """Checks the directives at the start of every step (between steps, nothing in flight)."""

    def __init__(self, rank: int, spec: Optional[str] = None) -> None:
        self.rank = rank
        self.faults = [f for f in parse_faults(os.environ.get("ZB_FAULT") if spec is None else spec) if f.rank == rank]

    def __bool__(self) -> bool:
        return bool(self.faults)

    def at_step(self, step: int, collectives=None) -> None:
        for f in self.faults:
            if f.step != step:
                continue
            print(f"[fault] rank {self.rank}: injecting {f.kind} at step {step}", file=sys.stderr, flush=True)
            if f.kind == "skip_signal":
                arm = getattr(collectives, "skip_next_collective", None)
                if arm is None:
                    raise ValueError("skip_signal needs the NVLink collectives (--collective-impl nvls|p2p)")
                arm()
                continue
            if f.kind == "kill_rank":
                os._exit(int(os.environ.get("ZB_FAULT_EXIT_CODE", "43")))
            if f.kind == "raise_rank":
                raise FaultInjected(f"injected fault on rank {self.rank} at step {step}")
            time.sleep(float(os.environ.get("ZB_FAULT_STALL_S", "3600")))
