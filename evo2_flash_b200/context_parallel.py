"""Context-parallel prefill of one long sequence across the GPUs of a node.

Rank r of P holds the contiguous token slice [r L, (r+1) L) of the sequence
and runs every Hyena layer on it with the full weights; the exchange per layer
is a few MB instead of a (T, H) all-reduce:

  FIR layers (HCS K=7, HCM K=128)  the output of a token depends on the K+1
      tokens before it (K=3 short filter, then the K-tap inner FIR), so a rank
      prepends the last K+1 hidden rows of the previous slice (the "halo") as
      a fresh segment and drops the halo's outputs: exact, no collective.
  LI layer (HCL, order-16 modal SSM)  the state entering slice r depends on
      every earlier token.  Pass 1 runs the slice from a zero modal state (the
      short-filter window seeded from the 2-row halo) and leaves the slice's
      own final state A_r; one all-gather of the (H, 16) A_q; the state entering
      slice r is S_r = p^L S_{r-1} + A_{r-1} (S_0 = 0), the segment continuation
      of the reference (mixers.py:204-209, st += p^L s_prev) applied slice by
      slice; pass 2 reruns the slice from S_r (slice 0 starts from zero: its
      pass 1 is final).

in_proj and out_proj run once per slice.  The halo comes from the caller (in a
pipeline, the previous rank sends its last K+1 input rows).  The reference has
no context parallelism; this is the B200-side scaling path for long prefills.
"""

from __future__ import annotations

from types import SimpleNamespace

import torch
import torch.distributed as dist

from .forward_context import set_forward_metadata


def halo_rows(mixer) -> int:
    """Input rows of the previous slice that this layer's first token depends on."""
    if mixer.kind == "fir":
        return mixer.k_inner - 1 + mixer.k_short - 1
    return mixer.k_short - 1


def _segment_meta(n, device, init):
    return SimpleNamespace(
        num_decodes=0, num_decode_tokens=0, num_prefills=1, num_prefill_tokens=n,
        query_start_loc_p=torch.tensor([0, n], dtype=torch.int32, device=device),
        has_initial_states_p=torch.tensor([init], dtype=torch.bool, device=device),
        state_indices_tensor_p=torch.tensor([1], dtype=torch.int32, device=device),
        state_indices_tensor_d=torch.zeros(0, dtype=torch.int32, device=device),
        query_start_loc_d=None, num_accepted_tokens=None,
        seq_lens=torch.tensor([n], dtype=torch.int32, device=device))


def li_entry_state(finals: torch.Tensor, log_poles: torch.Tensor, slice_lens, rank: int
                   ) -> torch.Tensor:
    """State entering slice `rank` from every slice's zero-start final state.

    finals (P, H, S) fp32: A_q; log_poles (H, S[, 1]); slice_lens: the token
    count of every slice (a sequence of P ints, or one int when all are equal).
    S_r = p^(L_{r-1}) S_{r-1} + A_{r-1}, S_0 = 0, with p^L = exp(L log p) in fp32:
    the state leaving slice q is its own A_q plus the entering state carried
    over that slice's own length."""
    P = finals.shape[0]
    lens = [int(slice_lens)] * P if isinstance(slice_lens, int) else [int(n) for n in slice_lens]
    if len(lens) != P:
        raise ValueError(f"{len(lens)} slice lengths for {P} slices")
    lp = log_poles.reshape(finals.shape[1], finals.shape[2]).float()
    s = torch.zeros_like(finals[0])
    for q in range(rank):
        s = torch.exp(lp * float(lens[q])) * s + finals[q]
    return s


def pack_final(final: torch.Tensor, slice_len: int) -> torch.Tensor:
    """(H + 1, S): a slice's final state with its token count in the extra row,
    so that one all-gather carries both (the count is exact in fp32 below 2^24)."""
    row = torch.full((1, final.shape[1]), float(slice_len), dtype=final.dtype,
                     device=final.device)
    return torch.cat([final, row])


def unpack_finals(packed: torch.Tensor):
    """(P, H + 1, S) gathered pack_final rows -> ((P, H, S) finals, [L_q])."""
    return packed[:, :-1], [int(v) for v in packed[:, -1, 0].tolist()]


def dist_gather(group=None):
    """gather(t) -> (P, ...) over a torch.distributed group (all-gather)."""
    def gather(t):
        ws = dist.get_world_size(group)
        buf = torch.empty((ws,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(buf, t.contiguous(), group=group)
        return buf
    return gather


class LiSlice:
    """An LI layer's slice between the two passes: `local_final` (H + 1, S) is
    A_r with this slice's token count in its last row (pack_final), to be
    gathered over the ranks; finish(gathered) runs pass 2."""

    def __init__(self, mixer, zl, meta, window, rank, g):
        self.mixer, self.zl, self.meta, self.window, self.rank = mixer, zl, meta, window, rank
        conv, inner = mixer._states_for_kernels()
        self.local_final = pack_final(inner[1, :, :mixer.state_size], zl.shape[0])
        # slice 0 enters with the zero state: its pass 1 is already exact
        self._out = mixer._out_proj(g) if rank == 0 else None

    def finish(self, gathered: torch.Tensor) -> torch.Tensor:
        if self._out is not None:
            return self._out
        m = self.mixer
        finals, lens = unpack_finals(gathered)
        if lens[self.rank] != self.zl.shape[0]:
            raise RuntimeError(f"slice {self.rank}: gathered length {lens[self.rank]} != "
                               f"{self.zl.shape[0]} (ranks gathered out of order)")
        conv, inner = m._states_for_kernels()
        with torch.no_grad():
            conv[1, :2] = self.window
            inner[1, :, :m.state_size] = li_entry_state(finals, m.log_poles, lens, self.rank)
        g = m._run_core(self.zl, self.meta, None)  # pass 2: from S_r -> exact outputs
        return m._out_proj(g)


def cp_prefill_start(mixer, x_local: torch.Tensor, x_halo: torch.Tensor | None, rank: int):
    """First half of cp_prefill: a FIR layer's outputs (L, H), or an LiSlice."""
    if mixer.tp_size != 1:
        raise ValueError("context-parallel prefill runs every layer unsharded (tp_size == 1)")
    dev = x_local.device
    L = x_local.shape[0]
    hr = halo_rows(mixer)
    first = x_halo is None
    if first != (rank == 0):
        raise ValueError("rank 0 takes no halo; every other rank needs one")
    if not first and x_halo.shape[0] < hr:
        raise ValueError(f"halo has {x_halo.shape[0]} rows, this layer needs {hr}")
    x_in = x_local if first else torch.cat([x_halo[-hr:], x_local])
    if mixer.kind == "fir":
        with set_forward_metadata(_segment_meta(x_in.shape[0], dev, False)):
            out = mixer(x_in)
        return out[x_in.shape[0] - L:]
    conv, inner = mixer._states_for_kernels()
    z = mixer._project(x_in)
    with torch.no_grad():
        if first:
            conv[1, :2].zero_()
        else:
            conv[1, :2] = z[:2]
        window = conv[1, :2].clone()
        inner[1, :, :mixer.state_size].zero_()
    zl = z[z.shape[0] - L:]
    meta = _segment_meta(L, dev, True)
    g = mixer._run_core(zl, meta, None)  # pass 1: from a zero modal state -> A_r
    return LiSlice(mixer, zl, meta, window, rank, g)


def cp_prefill(mixer, x_local: torch.Tensor, x_halo: torch.Tensor | None, rank: int,
               gather=None) -> torch.Tensor:
    """This rank's outputs (L, H) for its slice of one sequence.

    mixer: a HyenaFIRMixer / HyenaIIRMixer with tp_size == 1 whose kv_cache has
    at least 2 blocks (block 1 holds this slice's state; on return it is the
    state after the slice, as after an ordinary prefill).  x_local (L, H):
    this slice's hidden states; x_halo: the previous slice's last rows (at
    least halo_rows(mixer); None on rank 0).  gather(t) -> (P, ...) stacks a
    tensor over the ranks in rank order (default: dist_gather()); the LI layer
    calls it once on every rank.  Slices may differ in length: each rank's
    token count travels with its final state in the one all-gather."""
    r = cp_prefill_start(mixer, x_local, x_halo, rank)
    if isinstance(r, torch.Tensor):
        return r
    return r.finish((gather or dist_gather())(r.local_final))
