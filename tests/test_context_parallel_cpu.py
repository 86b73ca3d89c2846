"""The LI slice-state combination of context-parallel prefill, on CPU: the
state entering slice r, built from every slice's zero-start final state, equals
running the modal recurrence s = p s + u over all earlier tokens."""

import torch


def test_entry_state_equals_sequential_recurrence():
    from evo2_flash_b200.context_parallel import li_entry_state

    H, S, P, L = 6, 16, 5, 37
    g = torch.Generator().manual_seed(3)
    lp = -torch.exp(torch.rand(H, S, 1, generator=g) * 6 - 6)
    p = lp[..., 0].double().exp()
    u = torch.randn(P * L, H, generator=g).double()
    finals, entry, s = [], [], torch.zeros(H, S, dtype=torch.float64)
    for r in range(P):
        entry.append(s.clone())
        a = torch.zeros(H, S, dtype=torch.float64)
        for t in range(r * L, (r + 1) * L):
            a = a * p + u[t][:, None]
            s = s * p + u[t][:, None]
        finals.append(a)
    finals = torch.stack(finals).float()
    for r in range(P):
        got = li_entry_state(finals, lp, L, r)
        assert torch.allclose(got.double(), entry[r], rtol=1e-4, atol=1e-4), r


def test_entry_state_with_unequal_slices():
    """Slices of different lengths: each earlier slice carries the entering
    state over its own length (the count travels in the gathered tensor)."""
    from evo2_flash_b200.context_parallel import li_entry_state, pack_final, unpack_finals

    H, S = 5, 16
    lens = [11, 40, 3, 25]
    g = torch.Generator().manual_seed(4)
    lp = -torch.exp(torch.rand(H, S, 1, generator=g) * 6 - 6)
    p = lp[..., 0].double().exp()
    u = torch.randn(sum(lens), H, generator=g).double()
    packed, entry, s, t0 = [], [], torch.zeros(H, S, dtype=torch.float64), 0
    for n in lens:
        entry.append(s.clone())
        a = torch.zeros(H, S, dtype=torch.float64)
        for t in range(t0, t0 + n):
            a = a * p + u[t][:, None]
            s = s * p + u[t][:, None]
        packed.append(pack_final(a.float(), n))
        t0 += n
    finals, got_lens = unpack_finals(torch.stack(packed))
    assert got_lens == lens
    for r in range(len(lens)):
        got = li_entry_state(finals, lp, got_lens, r)
        assert torch.allclose(got.double(), entry[r], rtol=1e-4, atol=1e-4), r
