"""Host-side bounds checks of data-dependent indices (debug mode).

With ``AFD_BOUNDS_CHECK=1`` the op layer copies the MoE routing tables that
the routing kernels produce (moe_gate / moe_route / moe_align) back to the
host after each routing step and validates every index the grouped GEMMs,
the gather and the combine will dereference, before those kernels run. A
violation raises ``AFDBoundsError`` naming the first bad entry instead of
letting a kernel read or write out of range. This costs a device
synchronisation per MoE layer and is skipped while a CUDA graph is being
captured; it replaces the device sanitizer, which is not available here.

Invariants of one routing result (T tokens, top-k ids each, experts
[expert_start, expert_start + n_local) on this rank):

* ``num_rows`` = the number of (token, slot) pairs routed to a local expert;
  ``expert_offsets`` is an exclusive prefix sum of the per-expert counts;
* ``inv[t*k + j]`` is -1 for a non-local expert, else a row inside that
  expert's range, and the local rows form a permutation of [0, num_rows);
* ``row_token[row] = t`` and ``row_weight[row] = weights[t, j]``;
* ``blocks[:num_blocks]`` = {row_start, n_rows, expert, 0} cover every
  expert's rows in order, in pieces of at most ``block_n`` rows.
"""

from __future__ import annotations

import torch


class AFDBoundsError(RuntimeError):
    """A data-dependent index is outside the buffer it addresses."""


def _fail(msg: str) -> None:
    raise AFDBoundsError(msg)


def check_routing_tables(ids: torch.Tensor, weights: torch.Tensor, expert_start: int,
                         n_local: int, block_n: int, inv: torch.Tensor, row_token: torch.Tensor,
                         row_weight: torch.Tensor, expert_offsets: torch.Tensor,
                         blocks: torch.Tensor, num_blocks: torch.Tensor,
                         num_rows: torch.Tensor) -> None:
    """Validate one routing result (see the module docstring); raises
    AFDBoundsError on the first violation."""
    ids = ids.detach().to("cpu", torch.int64)
    T, k = ids.shape
    w = weights.detach().float().cpu().reshape(T * k)
    flat = ids.reshape(-1)
    inv = inv.detach().to("cpu", torch.int64)[: T * k]
    n_rows = int(num_rows.reshape(-1)[0])
    n_blk = int(num_blocks.reshape(-1)[0])
    offs = expert_offsets.detach().to("cpu", torch.int64)[: n_local + 1]
    local = flat - expert_start
    is_local = (local >= 0) & (local < n_local)
    if bool(((flat < 0)).any()):
        _fail(f"negative expert id at entry {int((flat < 0).nonzero()[0])}")
    want_rows = int(is_local.sum())
    if n_rows != want_rows:
        _fail(f"num_rows {n_rows} != {want_rows} locally routed pairs")
    if n_rows > row_token.numel():
        _fail(f"num_rows {n_rows} exceeds the row buffers ({row_token.numel()})")
    counts = torch.bincount(local[is_local], minlength=n_local)
    want_offs = torch.cat([torch.zeros(1, dtype=torch.int64), counts.cumsum(0)])
    if not torch.equal(offs, want_offs):
        bad = int((offs != want_offs).nonzero()[0])
        _fail(f"expert_offsets[{bad}] = {int(offs[bad])}, expected {int(want_offs[bad])}")
    if bool((inv[~is_local] != -1).any()):
        bad = int(((inv != -1) & ~is_local).nonzero()[0])
        _fail(f"inv[{bad}] = {int(inv[bad])} for a non-local expert (expected -1)")
    li = is_local.nonzero().reshape(-1)
    rows = inv[li]
    e = local[li]
    lo, hi = offs[e], offs[e + 1]
    out = (rows < lo) | (rows >= hi)
    if bool(out.any()):
        j = int(li[out.nonzero()[0]])
        _fail(f"inv[{j}] = {int(inv[j])} outside expert {int(local[j])}'s rows "
              f"[{int(offs[local[j]])}, {int(offs[local[j] + 1])})")
    if rows.numel() and torch.unique(rows).numel() != rows.numel():
        _fail("two routed pairs share a row")
    rt = row_token.detach().to("cpu", torch.int64)[:n_rows]
    rw = row_weight.detach().float().cpu()[:n_rows]
    tok = li // k
    if not torch.equal(rt[rows], tok):
        j = int(li[(rt[rows] != tok).nonzero()[0]])
        _fail(f"row_token[{int(inv[j])}] = {int(rt[inv[j]])}, expected token {j // k}")
    if not torch.equal(rw[rows], w[li]):
        j = int(li[(rw[rows] != w[li]).nonzero()[0]])
        _fail(f"row_weight[{int(inv[j])}] does not hold the routing weight of entry {j}")
    b = blocks.detach().to("cpu", torch.int64).reshape(-1, 4)
    if n_blk > b.shape[0]:
        _fail(f"num_blocks {n_blk} exceeds the block list ({b.shape[0]})")
    b = b[:n_blk]
    nxt = torch.zeros(n_local, dtype=torch.int64) + offs[:-1]
    last_e = -1
    for i in range(n_blk):
        start, n, ex = int(b[i, 0]), int(b[i, 1]), int(b[i, 2])
        if not 0 <= ex < n_local:
            _fail(f"block {i}: expert {ex} outside [0, {n_local})")
        if ex < last_e:
            _fail(f"block {i}: experts out of order ({ex} after {last_e})")
        if not 0 < n <= block_n:
            _fail(f"block {i}: {n} rows (block size {block_n})")
        if start != int(nxt[ex]) or start + n > int(offs[ex + 1]):
            _fail(f"block {i}: rows [{start}, {start + n}) do not continue expert {ex}'s "
                  f"range [{int(offs[ex])}, {int(offs[ex + 1])}) at {int(nxt[ex])}")
        nxt[ex] = start + n
        last_e = ex
    if not torch.equal(nxt, offs[1:]):
        ex = int((nxt != offs[1:]).nonzero()[0])
        _fail(f"blocks cover expert {ex}'s rows only up to {int(nxt[ex])} of {int(offs[ex + 1])}")
