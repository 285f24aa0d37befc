"""N-sharded gate/up: the prefix LM's MLP split over P GPUs (one process each).

The reference runs on one GPU and has no counterpart; this is the optional
tensor-parallel variant of the W4A4 path.  Every rank runs the same
observations through the attention block (replicated), then:

1. rank p holds rows [p N/P, (p+1) N/P) of gate_proj and up_proj and computes
   those columns of gate and up for all M tokens (one W4A4 GEMM launch), and
   their GeGLU;
2. the ranks exchange row blocks of that [M, N/P] result with one NCCL
   all-to-all, so that rank p receives, for its M/P tokens, the P column
   segments that make up their full 16384-wide rows -- P times fewer bytes
   than an all-gather of h to every rank;
3. rank p quantises its M/P complete rows straight from the received
   segments (w4a4_quant_segments: a 4-D TMA box per row, no transpose) and
   runs down_proj on them;
4. an NCCL all-gather of the [M/P, hidden] down_proj outputs restores the
   full residual stream on every rank.

The results are bit-identical to the one-GPU forward: every output element of
a W4A4 GEMM depends only on its row and column, the exchanges copy bits, and
the quant sees the same row values.  down_proj cannot be split by K instead:
its activation quant is a Hadamard rotation and an amax over the whole
16384-wide row.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class MlpShard:
    """This process's place in the tensor-parallel MLP."""

    rank: int
    world: int
    group: object = None  # torch.distributed process group (None: the default group)

    def cols(self, n: int) -> slice:
        """Rows of gate_proj / up_proj (columns of gate / up) this rank holds."""
        if n % self.world:
            raise ValueError(f"MLP width {n} is not divisible by {self.world} ranks")
        w = n // self.world
        return slice(self.rank * w, (self.rank + 1) * w)

    def rows(self, m: int) -> slice:
        """Token rows whose down_proj this rank computes."""
        if m % self.world:
            raise ValueError(f"{m} token rows are not divisible by {self.world} ranks")
        r = m // self.world
        return slice(self.rank * r, (self.rank + 1) * r)


def exchange_row_blocks(part: torch.Tensor, recv: torch.Tensor, shard: MlpShard) -> torch.Tensor:
    """part [M, n] (this rank's columns of every row) -> recv [P, M/P, n]:
    recv[q] = rank q's columns of this rank's M/P rows.  Row block q of
    `part` is contiguous, so one all-to-all with equal splits does it."""
    if not part.is_contiguous() or not recv.is_contiguous() or recv.numel() != part.numel():
        raise ValueError("exchange_row_blocks needs contiguous buffers of equal size")
    dist.all_to_all_single(recv.view(-1), part.view(-1), group=shard.group)
    return recv


def gather_row_blocks(part: torch.Tensor, out: torch.Tensor, shard: MlpShard) -> torch.Tensor:
    """part [M/P, h] of every rank -> out [M, h] on every rank (rank order =
    row order)."""
    dist.all_gather_into_tensor(out, part, group=shard.group)
    return out
