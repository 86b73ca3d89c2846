"""The decode plan (evo2_flash_b200.mixers.plan_decode) on CPU: which blocks
each decode request reads and writes, from the engine metadata alone.  The
expected tables below are written out from the slot rules of the reference's
verifier (mixers.py:443-540): column p of a request's block table is the
snapshot slot of verifier position p; in prefix-caching "all" mode the window
starts at the request's last scheduled block (inputs: the previous step's);
a table that cannot fit the state cache (vLLM's profiling pass) points at the
null block."""

from types import SimpleNamespace

import pytest
import torch

from evo2_flash_b200.mixers import plan_decode


def _meta(table, tokens=None, starts=None, **kw):
    reqs = table.shape[0]
    return SimpleNamespace(num_decodes=reqs, num_decode_tokens=tokens or reqs,
                           state_indices_tensor_d=table, query_start_loc_d=starts, **kw)


def test_single_token_table():
    t = torch.tensor([5, 7, 9], dtype=torch.int32)
    p = plan_decode(_meta(t), 1, 64)
    assert p.reqs == 3 and p.starts is None and p.engine_accepted is None
    assert p.in_slots.tolist() == [[5], [7], [9]]
    assert p.out_slots.tolist() == [[5], [7], [9]]
    assert p.conv_in.tolist() == [5, 7, 9] and p.conv_out.tolist() == [5, 7, 9]


def test_speculative_table_and_engine_counts():
    t = torch.tensor([[1, 2, 3, 4, 40], [5, 6, 7, 8, 41]], dtype=torch.int32)
    starts = torch.tensor([0, 4, 6, 99], dtype=torch.int32)
    acc = torch.tensor([0, 3, 2])
    p = plan_decode(_meta(t, 6, starts, num_accepted_tokens=acc), 4, 64)
    assert p.in_slots.tolist() == [[1, 2, 3, 4], [5, 6, 7, 8]]  # width = positions
    assert p.starts.tolist() == [0, 4, 6]
    assert p.engine_accepted.tolist() == [0, 3]  # cut to the requests (kernels read 0 as 1)
    assert p.conv_in.tolist() == [1, 5]


def test_prefix_caching_window_moves_along_the_table():
    t = torch.arange(1, 13, dtype=torch.int32).view(2, 6)
    m = _meta(t, 8, torch.tensor([0, 4, 8], dtype=torch.int32),
              block_idx_last_scheduled_token_prev_step=torch.tensor([0, 1]),
              block_idx_last_scheduled_token=torch.tensor([2, 1]),
              block_idx_last_computed_token=torch.tensor([1, 0]))
    p = plan_decode(m, 4, 64)
    assert p.in_slots.tolist() == [[1, 2, 3, 4], [8, 9, 10, 11]]
    assert p.out_slots.tolist() == [[3, 4, 5, 6], [8, 9, 10, 11]]
    assert p.conv_in.tolist() == [2, 7] and p.conv_out.tolist() == [3, 8]


def test_profiling_table_points_at_the_null_block():
    t = torch.arange(1, 9, dtype=torch.int32).view(2, 4)
    p = plan_decode(_meta(t, 8, torch.tensor([0, 4, 8], dtype=torch.int32)), 4, 2)
    assert not p.in_slots.any() and not p.out_slots.any() and not p.conv_in.any()
    assert not p.table.any()


def test_shape_errors_raise_value_error():
    with pytest.raises(ValueError):
        plan_decode(_meta(torch.zeros(2, 2, 2, dtype=torch.int32)), 1, 8)
    m = _meta(torch.tensor([1, 2], dtype=torch.int32))
    m.num_decodes = 3
    with pytest.raises(ValueError):
        plan_decode(m, 1, 8)
    with pytest.raises(ValueError):  # several tokens per request without offsets
        plan_decode(_meta(torch.tensor([[1, 2], [3, 4]], dtype=torch.int32), 4), 2, 8)
    with pytest.raises(ValueError):
        plan_decode(_meta(torch.tensor([[1, 2]], dtype=torch.int32), 2,
                          torch.tensor([0], dtype=torch.int32)), 2, 8)
    with pytest.raises(ValueError):
        plan_decode(_meta(torch.tensor([1, 2], dtype=torch.int32),
                          num_accepted_tokens=torch.tensor([1])), 1, 8)
