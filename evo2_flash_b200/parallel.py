"""Channel-group sharding of a Hyena mixer across the GPUs of one node.

Every operation between the two projections is per channel (depthwise FIRs,
elementwise gates, a diagonal SSM), so rank r of P owns channels
[r*H/P, (r+1)*H/P):

  in_proj    rows [3 r H/P, 3 (r+1) H/P) of the interleaved (3H, H) weight: whole
             (x2, x1, v) triples (mixers.py:1207-1208), so each rank's z is the
             in_proj output of its own channels (column-parallel, no exchange);
  short_filter  the same rows; conv, D, log_poles, residues: rows [r H/P, ...);
  out_proj   columns [r H/P, (r+1) H/P) (row-parallel): each rank produces a
             partial (T, H) sum, one all-reduce completes it, the bias is added
             once afterwards;
  paged state  each rank holds its own channels' slices (S0 (., 3H/P), S1 (., H/P),
             S2 (H/P, .)), exactly the shrunken spec vLLM derives for TP.

The reference has no tensor parallelism (mixers.py:38-41); this is the
B200-side addition for the 40B shape.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def channel_slice(hidden: int, rank: int, world: int) -> slice:
    if hidden % world:
        raise ValueError(f"hidden size {hidden} does not split over {world} ranks")
    h = hidden // world
    return slice(h * rank, h * (rank + 1))


def shard_mixer_tensors(tensors: dict, rank: int, world: int, hidden: int) -> dict:
    """This rank's shard of one Hyena layer's unsharded tensors (checkpoint names)."""
    rows = channel_slice(hidden, rank, world)
    rows3 = slice(3 * rows.start, 3 * rows.stop)
    out = {}
    for name, t in tensors.items():
        if name == "in_proj.weight":
            out[name] = t[rows3]
        elif name == "short_filter":
            out[name] = t.reshape(3 * hidden, 1, -1)[rows3]
        elif name == "out_proj.weight":
            out[name] = t[:, rows]
        elif name in ("in_proj.weight_scale", "in_proj.input_scale", "out_proj.bias"):
            out[name] = t
        elif name == "conv":
            out[name] = t.reshape(hidden, 1, -1)[rows]
        elif name in ("D", "residues"):
            out[name] = t[rows]
        elif name == "log_poles":
            out[name] = t.reshape(hidden, -1, 1)[rows]
        elif name in ("in_proj_token_table", "in_proj_emul_weight_t", "in_proj_emul_scales",
                      "in_proj_emul_cols"):
            if world != 1:  # FP8-surgery projections (mixers.py:758-800)
                raise ValueError(f"{name}: FP8-surgery layers are not channel-sharded")
            out[name] = t
        else:
            raise KeyError(f"unexpected mixer tensor {name!r}")
    return out


def all_reduce_partial(out: torch.Tensor, bias: torch.Tensor | None, group=None) -> torch.Tensor:
    """Completes a row-parallel out_proj: sum the ranks' partials, add the bias once."""
    dist.all_reduce(out, group=group)
    return out if bias is None else out + bias


class PendingReduce:
    """A row-parallel out_proj whose all-reduce is in flight (NCCL runs on its
    own stream).  `wait()` orders the caller's current stream after the reduce,
    adds the bias once and returns the completed output; until then the caller
    may launch other work (the next chunk or layer), which the reduce overlaps."""

    def __init__(self, out, bias, work, finish=None):
        self._out, self._bias, self._work, self._finish = out, bias, work, finish
        self._done = None

    def wait(self) -> torch.Tensor:
        if self._done is None:
            if self._work is not None:
                self._work.wait()
            out = self._out if self._bias is None else self._out + self._bias
            self._done = self._finish(out) if self._finish is not None else out
        return self._done


def all_reduce_partial_async(out: torch.Tensor, bias: torch.Tensor | None, group=None,
                             finish=None) -> PendingReduce:
    """all_reduce_partial with the collective left in flight (see PendingReduce)."""
    work = dist.all_reduce(out, group=group, async_op=True)
    return PendingReduce(out, bias, work, finish)
