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


class PendingNvls:
    """A row-parallel out_proj whose in-switch all-reduce runs on the reducer's
    collective stream; wait() orders the caller's stream after it and returns
    the reduced rows (a view into the reducer's buffer ring, valid until `slots`
    further reductions have been started)."""

    def __init__(self, out, done, finish=None):
        self._out, self._ev, self._finish = out, done, finish
        self._done = None

    def wait(self) -> torch.Tensor:
        if self._done is None:
            torch.cuda.current_stream().wait_event(self._ev)
            self._done = self._finish(self._out) if self._finish is not None else self._out
        return self._done


class NvlsReducer:
    """In-switch (NVLink SHARP) all-reduce of row-parallel partial sums for one
    process group (hyena_nvls_allreduce_bf16).

    The out_proj GEMM of every rank writes its partial straight into the next
    buffer of a ring of symmetric, multicast-mapped buffers; the reduction
    kernel then runs on a high-priority collective stream with a few CTAs, so
    it proceeds beside the next layer's or chunk's kernels instead of taking
    whole SMs the way a ring all-reduce does.  A buffer is written again only
    after this rank's previous reduction of it has finished, which (through the
    kernel's closing handshake) means every rank has finished with it too.
    Every rank must make the same calls in the same order."""

    def __init__(self, group, max_elems: int, device, slots: int = 32, num_ctas: int = 16):
        import torch.distributed._symmetric_memory as symm

        self.group = group if group is not None else dist.group.WORLD
        self.max_elems = (int(max_elems) + 7) // 8 * 8
        self.slots, self.num_ctas = slots, num_ctas
        self.buf = symm.empty((slots, self.max_elems), dtype=torch.bfloat16, device=device)
        self.hdl = symm.rendezvous(self.buf, self.group.group_name)
        if not self.hdl.multicast_ptr:
            raise RuntimeError("NVLink multicast is not available for this group")
        self.rank, self.world = self.hdl.rank, self.hdl.world_size
        self.stream = torch.cuda.Stream(device=device, priority=-1)
        self.epoch = 0
        self.next = 0
        self.done = [None] * slots
        self.error = torch.zeros(1, dtype=torch.int32, device=device)

    def buffer(self, rows: int, cols: int):
        """The next ring buffer as a (rows, cols) bf16 tensor, once this rank's
        previous reduction of it has finished."""
        n = rows * cols
        if n > self.max_elems:
            raise ValueError(f"{n} elements exceed the reducer's {self.max_elems}")
        k = self.next
        self.next = (k + 1) % self.slots
        if self.done[k] is not None:
            torch.cuda.current_stream().wait_event(self.done[k])
        return k, self.buf[k, :n].view(rows, cols)

    def reduce_async(self, k: int, t: torch.Tensor, finish=None) -> PendingNvls:
        """Starts the all-reduce of ring buffer k (holding t) after the caller's
        stream has produced it."""
        from . import _lib

        ready = torch.cuda.Event()
        ready.record()
        self.stream.wait_event(ready)
        self.epoch += 1
        n = t.numel()
        n_pad = (n + 7) // 8 * 8
        mc = self.hdl.multicast_ptr + k * self.max_elems * 2
        _lib.check(_lib.load().hyena_nvls_allreduce_bf16(
            _lib.C.c_void_p(mc), n_pad, _lib.C.c_void_p(self.hdl.signal_pad_ptrs_dev),
            self.hdl.signal_pad_size, self.rank, self.world, self.epoch, self.num_ctas,
            _lib.C.c_void_p(self.error.data_ptr()), _lib.C.c_void_p(self.stream.cuda_stream)),
            "hyena_nvls_allreduce_bf16")
        done = torch.cuda.Event()
        done.record(self.stream)
        self.done[k] = done
        return PendingNvls(t, done, finish)

    def check(self) -> None:
        """Raises if a cross-rank wait of an earlier reduction expired (reads the
        device error word: synchronises with the collective stream)."""
        self.stream.synchronize()
        if int(self.error.item()):
            raise RuntimeError("NVLS all-reduce: a cross-rank wait expired (ranks out of step)")


_REDUCERS: dict = {}


def nvls_reducer(group, elems: int, device, slots: int = 32):
    """The process-wide NvlsReducer of (group, device), grown to hold `elems`
    per buffer (growing re-allocates: a collective call, made by every rank at
    the same point because every rank runs the same layers), or None when the
    group's GPUs have no NVLink multicast."""
    key = (id(group), str(device))
    red = _REDUCERS.get(key)
    if red is False:
        return None
    if red is None or red.max_elems < elems:
        try:
            red = NvlsReducer(group, max(elems, 0 if red is None else red.max_elems), device, slots)
        except RuntimeError:
            _REDUCERS[key] = False
            return None
        _REDUCERS[key] = red
    return red
