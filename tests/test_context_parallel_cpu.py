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
