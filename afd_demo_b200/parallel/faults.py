"""Host-side fault injection, driven by the ``AFD_FAULT`` environment variable.

The reference has no fault injection and no failure detection beyond the
experiment scripts' OOM grep (scripts/run_single.sh:342-348) and an EXIT trap
that kills the background FFN process (scripts/run_single.sh:226-233). Faults
here are made on the host only -- an exception, a process exit, a message
that is not sent, a delay -- so that the detection paths can be exercised on
CPU ranks (gloo) or on GPUs without corrupting device state.

``AFD_FAULT`` is a comma-separated list of items:

    oom                   raise an out-of-memory error while the model loads
    raise_rank:R[:S]      rank R raises before decode step S (default 0)
    exit_rank:R[:S]       rank R leaves without cleanup (exit code 17) before
                          decode step S, after reporting nothing
    drop:D:L[:M]          the host transport skips direction D's (a2f | f2a)
                          send of layer L, micro-batch M (default 0), once
    delay_ms:N[:R]        rank R (every rank if absent) sleeps N ms before
                          each decode step
"""

from __future__ import annotations

import os
import time
from dataclasses import dataclass, field
from typing import Dict, Optional, Set, Tuple

import torch


class InjectedFault(RuntimeError):
    """Raised by an injected ``raise_rank`` fault."""


@dataclass
class FaultPlan:
    oom: bool = False
    raise_at: Dict[int, int] = field(default_factory=dict)   # rank -> step
    exit_at: Dict[int, int] = field(default_factory=dict)    # rank -> step
    drops: Set[Tuple[str, int, int]] = field(default_factory=set)
    delay_ms: float = 0.0
    delay_rank: Optional[int] = None

    @classmethod
    def parse(cls, spec: Optional[str]) -> "FaultPlan":
        plan = cls()
        for item in filter(None, (s.strip() for s in (spec or "").split(","))):
            parts = item.split(":")
            kind = parts[0]
            try:
                if kind == "oom":
                    plan.oom = True
                elif kind in ("raise_rank", "exit_rank"):
                    r, s = int(parts[1]), int(parts[2]) if len(parts) > 2 else 0
                    (plan.raise_at if kind == "raise_rank" else plan.exit_at)[r] = s
                elif kind == "drop":
                    d = parts[1]
                    if d not in ("a2f", "f2a"):
                        raise ValueError(d)
                    plan.drops.add((d, int(parts[2]), int(parts[3]) if len(parts) > 3 else 0))
                elif kind == "delay_ms":
                    plan.delay_ms = float(parts[1])
                    plan.delay_rank = int(parts[2]) if len(parts) > 2 else None
                else:
                    raise ValueError(kind)
            except (IndexError, ValueError) as e:
                raise ValueError(f"bad AFD_FAULT item {item!r}") from e
        return plan

    @property
    def active(self) -> bool:
        return bool(self.oom or self.raise_at or self.exit_at or self.drops or self.delay_ms)

    # ------------------------------------------------------------ hooks
    def on_load(self) -> None:
        if self.oom:
            raise torch.OutOfMemoryError("injected out-of-memory (AFD_FAULT=oom)")

    def before_step(self, rank: int, step: int) -> None:
        if self.delay_ms and (self.delay_rank is None or self.delay_rank == rank):
            time.sleep(self.delay_ms / 1000.0)
        if self.raise_at.get(rank) == step:
            raise InjectedFault(f"injected failure on rank {rank} before decode step {step}")
        if self.exit_at.get(rank) == step:
            os._exit(17)

    def drop(self, direction: str, layer: int, mb: int) -> bool:
        key = (direction, layer, mb)
        if key in self.drops:
            self.drops.discard(key)  # once
            return True
        return False


_PLAN: Optional[FaultPlan] = None


def plan() -> FaultPlan:
    """The process's fault plan (parsed from ``AFD_FAULT`` on first use)."""
    global _PLAN
    if _PLAN is None:
        _PLAN = FaultPlan.parse(os.environ.get("AFD_FAULT"))
    return _PLAN


def set_plan(p: Optional[FaultPlan]) -> None:
    """Replace the plan (tests); None re-reads the environment next time."""
    global _PLAN
    _PLAN = p
