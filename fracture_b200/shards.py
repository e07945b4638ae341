"""How the hot path's work is split over the GPUs of one box, and the one exchange it needs.

* Prefill chain: sequences are independent, so each rank runs its own
  sequences (``sequence_shard``) with no collective on the data path.
* TurboQuant KV cache (config 4): a sequence's token range is split at 16-token cache-block
  boundaries (``block_shard``); each rank owns a disjoint pool shard and block-table slice.
* Pipeline (config 5): stage ``s`` holds a contiguous run of layers (``stage_layers``); the
  hidden states of every micro-batch move from stage ``s`` to ``s + 1`` by point-to-point
  send/recv (``StageLink``, NCCL over NVLink on the box). This replaces the reference
  coordinator's handoff, which copies each stage's activations device-to-host, sends them over
  TCP and copies them host-to-device on the next worker, one stage at a time
  (``crates/fracture-coordinator/src/pipeline.rs:434-539``,
  ``bins/fracture-worker-cuda/src/main.rs:1350-1446``).

``max_over_ranks`` is the timing aggregate every multi-GPU figure uses. Everything here runs
unchanged on the ``gloo`` backend with CPU tensors (tests) and on ``nccl`` with CUDA tensors.
"""

from __future__ import annotations

from dataclasses import dataclass

BLOCK_TOKENS = 16  # tokens per paged-cache block (paged_kv_cache.rs:7)


def _even_split(n: int, world: int, rank: int) -> tuple[int, int]:
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def sequence_shard(n_seq: int, world: int, rank: int) -> range:
    """Sequences of this rank: contiguous, sizes differing by at most one."""
    start, count = _even_split(n_seq, world, rank)
    return range(start, start + count)


def block_shard(n_tokens: int, world: int, rank: int, block: int = BLOCK_TOKENS) -> range:
    """Token range of this rank, cut at multiples of ``block`` (the last rank takes the ragged end)."""
    n_blocks = (n_tokens + block - 1) // block
    b0, nb = _even_split(n_blocks, world, rank)
    return range(min(b0 * block, n_tokens), min((b0 + nb) * block, n_tokens))


def stage_layers(n_layers: int, world: int, rank: int) -> range:
    """Layers held by pipeline stage ``rank`` (contiguous; the first stages take the remainder)."""
    start, count = _even_split(n_layers, world, rank)
    return range(start, start + count)


def max_over_ranks(value: float, device=None) -> float:
    """Maximum of ``value`` over all ranks (the value itself without a process group)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


@dataclass
class StageLink:
    """Point-to-point links of pipeline stage ``rank``: receive from ``rank - 1``, send to
    ``rank + 1``; with ``ring`` the last stage also sends to stage 0 (decode feeds the next
    step's tokens back). Sends are asynchronous; a receive can be posted ahead of the compute
    it feeds."""

    rank: int
    world: int
    ring: bool = False

    @property
    def prev(self) -> int | None:
        if self.rank > 0:
            return self.rank - 1
        return self.world - 1 if self.ring and self.world > 1 else None

    @property
    def next(self) -> int | None:
        if self.rank < self.world - 1:
            return self.rank + 1
        return 0 if self.ring and self.world > 1 else None

    def isend(self, tensor):
        import torch.distributed as dist

        if self.next is None:
            raise RuntimeError(f"stage {self.rank} has no next stage")
        return dist.isend(tensor, self.next)

    def irecv(self, tensor):
        import torch.distributed as dist

        if self.prev is None:
            raise RuntimeError(f"stage {self.rank} has no previous stage")
        return dist.irecv(tensor, self.prev)


def run_pipeline(n_micro: int, link: StageLink, first_input, stage_fn, recv_buffers, on_output=None):
    """Forward-only micro-batched pipeline on this stage.

    Stage 0 takes micro-batch ``m`` from ``first_input(m)``; other stages receive it from the
    previous stage into ``recv_buffers[m % len(recv_buffers)]`` (the receive of ``m + 1`` is
    posted before ``m`` is computed). ``stage_fn(m, x)`` runs this stage's layers and returns the
    tensor to hand on; the send of ``m`` overlaps the compute of ``m + 1`` (at most one send in
    flight, so a result buffer may be reused two micro-batches later). A ``stage_fn`` that works in
    place and returns its input needs three receive buffers, so the receive of ``m + 1`` never
    lands in the buffer whose send (``m - 1``) may still be in flight. The last stage passes its
    results to ``on_output(m, y)``. Every stage posts the same sends and receives in the same
    order, so the links cannot deadlock.
    """
    first = link.prev is None or link.rank == 0
    last = link.next is None or link.rank == link.world - 1
    if not first and not recv_buffers:
        raise ValueError("a receiving stage needs at least one buffer")
    pending_recv = None
    if not first and n_micro > 0:
        pending_recv = link.irecv(recv_buffers[0])
    send_req = None
    for m in range(n_micro):
        if first:
            x = first_input(m)
        else:
            pending_recv.wait()
            x = recv_buffers[m % len(recv_buffers)]
            if m + 1 < n_micro:
                if len(recv_buffers) < 2:
                    raise ValueError("overlapping receives need two buffers")
                pending_recv = link.irecv(recv_buffers[(m + 1) % len(recv_buffers)])
        y = stage_fn(m, x)
        if not last:
            if send_req is not None:
                send_req.wait()
            send_req = link.isend(y)
        elif on_output is not None:
            on_output(m, y)
    if send_req is not None:
        send_req.wait()
