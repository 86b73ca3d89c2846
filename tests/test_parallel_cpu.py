"""Channel-group sharding (evo2_flash_b200.parallel) on CPU with gloo ranks.

Each rank runs the oracle mixer on its channel shard (its rows of in_proj as
whole triples, its filters, its slice of the paged state), produces the partial
out_proj sum of its columns, and one all-reduce plus the bias must reproduce the
unsharded mixer: prefill with continuation segments, then a decode step.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.helpers import (decode_meta, max_rel_err, params_to_oracle, prefill_meta,
                           random_params)

H = 128


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _states(h, nb=4):
    return [torch.zeros(nb, 2, 3 * h, dtype=torch.bfloat16), torch.zeros(nb, 127, h),
            torch.zeros(nb, h, 16)]


def _steps():
    g = torch.Generator().manual_seed(5)
    metas = [prefill_meta([40, 9], [1, 2], [False, False]),
             prefill_meta([12], [1], [True]),
             decode_meta([1, 2])]
    xs = [torch.randn(int(m.num_prefill_tokens) + int(m.num_decode_tokens), H, generator=g)
          .to(torch.bfloat16) for m in metas]
    return metas, xs


def _sharded_forward(rank, world, kind, k, port, results):
    from oracle import hyena_oracle as O
    from evo2_flash_b200.parallel import channel_slice, shard_mixer_tensors

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = random_params(kind, H, k, seed=17)
        shard = shard_mixer_tensors(full, rank, world, H)
        hl = H // world
        p = params_to_oracle(shard, kind, hl, k)
        bias = p.out_proj_bias
        p.out_proj_bias = None
        states = _states(hl)
        outs = []
        metas, xs = _steps()
        for meta, x in zip(metas, xs):
            z = O.in_proj(x, p)
            g = O.mixer_core(z, p, meta, states, None, bf16_products=True)
            part = (g.float() @ p.out_proj_weight.float().t())  # fp32 partial sum
            dist.all_reduce(part)
            outs.append((part + bias.float()).to(torch.bfloat16))
        if rank == 0:
            results["outs"] = outs
        sl = channel_slice(H, rank, world)
        results[f"s1_{rank}"] = states[1]
        results[f"s2_{rank}"] = states[2]
        results[f"rows_{rank}"] = (sl.start, sl.stop)
    finally:
        dist.destroy_process_group()


def _worker(rank, world, kind, k, port, out_dir):
    res = {}
    _sharded_forward(rank, world, kind, k, port, res)
    torch.save(res, os.path.join(out_dir, f"rank{rank}.pt"))


@pytest.mark.parametrize("kind,k", [("hcm", 128), ("hcl", 16)])
def test_channel_sharded_mixer_equals_unsharded(kind, k, tmp_path):
    from oracle import hyena_oracle as O

    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, kind, k, port, str(tmp_path)))
             for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=300)
        assert pr.exitcode == 0
    got = {}
    for r in range(world):
        got.update(torch.load(tmp_path / f"rank{r}.pt"))

    full = random_params(kind, H, k, seed=17)
    p = params_to_oracle(full, kind, H, k)
    states = _states(H)
    metas, xs = _steps()
    for i, (meta, x) in enumerate(zip(metas, xs)):
        ref = O.mixer_forward(x, p, meta, states, bf16_products=True)
        # one extra bf16 rounding (the reduce of fp32 partials vs one GEMM) at most
        assert max_rel_err(got["outs"][i], ref) < 1e-2, i
    for r in range(world):
        a, b = got[f"rows_{r}"]
        assert torch.equal(got[f"s1_{r}"], states[1][:, :, a:b])
        assert max_rel_err(got[f"s2_{r}"], states[2][:, a:b]) < 1e-6


def _async_worker(rank, world, port, out_dir):
    from evo2_flash_b200.parallel import all_reduce_partial_async

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(100 + rank)
        parts = [torch.randn(6, 8, generator=g) for _ in range(3)]
        bias = torch.arange(8, dtype=torch.float32)
        pend = [all_reduce_partial_async(p.clone(), bias, finish=lambda t: t[:5]) for p in parts]
        outs = [pr.wait() for pr in pend]
        assert all(pr.wait() is o for pr, o in zip(pend, outs))  # wait() is idempotent
        torch.save({"parts": parts, "outs": outs}, os.path.join(out_dir, f"a{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_async_all_reduce_completes_partials_once(tmp_path):
    """Several row-parallel reduces in flight at once; each wait() returns the
    sum over ranks plus the bias once, through the caller's finishing step."""
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_async_worker, args=(r, world, port, str(tmp_path)))
             for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=300)
        assert pr.exitcode == 0
    res = [torch.load(tmp_path / f"a{r}.pt") for r in range(world)]
    bias = torch.arange(8, dtype=torch.float32)
    for i in range(3):
        want = (res[0]["parts"][i] + res[1]["parts"][i] + bias)[:5]
        for r in range(world):
            assert torch.allclose(res[r]["outs"][i], want)
