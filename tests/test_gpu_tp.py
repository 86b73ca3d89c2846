"""Channel-sharded mixer modules on 2 GPUs: rank r owns half the channels (its
in_proj triples, filters and paged state), out_proj partial sums are all-reduced
-- by NCCL, or by the in-switch NVLS kernel (hyena_nvls_allreduce_bf16) -- and
every step must match the unsharded mixer on one GPU.  Skipped with fewer than 2
GPUs; the NVLS case also without NVLink multicast."""

import os
import socket
from types import SimpleNamespace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.helpers import (REL_TOL, decode_meta, max_rel_err, meta_to, prefill_meta,
                           random_params)

pytestmark = pytest.mark.gpu
H = 256


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _build(kind, k, dev, rank=0, world=1, group=None, collective="auto"):
    from evo2_flash_b200 import HyenaFIRMixer, HyenaIIRMixer

    cfg = SimpleNamespace(hidden_size=H, short_filter_length=3, hcm_filter_length=128,
                          state_size=16, use_fp8_input_projections=False)
    kw = dict(tp_rank=rank, tp_size=world, tp_group=group, device=dev, tp_collective=collective)
    m = (HyenaIIRMixer(cfg, 0, prefix="tp", **kw) if kind == "hcl"
         else HyenaFIRMixer(cfg, 0, prefix="tp", k_inner=k, **kw))
    m.load_full_weights({kk: v.to(dev) for kk, v in random_params(kind, H, k, seed=23).items()})
    m.allocate_state(4, dev)
    return m


def _steps():
    g = torch.Generator().manual_seed(24)
    metas = [prefill_meta([300, 77], [1, 2], [False, False]),
             prefill_meta([20], [1], [True]), decode_meta([1, 2]), decode_meta([1, 2])]
    xs = [torch.randn(int(m.num_prefill_tokens) + int(m.num_decode_tokens), H, generator=g)
          .to(torch.bfloat16) for m in metas]
    return metas, xs


def _run(m, dev):
    from evo2_flash_b200 import set_forward_metadata

    outs = []
    for meta, x in zip(*_steps()):
        with set_forward_metadata(meta_to(meta, dev)):
            outs.append(m(x.to(dev)).cpu())
    torch.cuda.synchronize()
    return outs


def _worker(rank, world, kind, k, port, out_dir, collective):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    from datetime import timedelta

    from evo2_flash_b200 import parallel

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=dev)
    try:
        if collective == "nvls" and parallel.nvls_reducer(dist.group.WORLD, 1 << 17, dev) is None:
            if rank == 0:
                torch.save("no multicast", os.path.join(out_dir, "tp.pt"))
        else:
            m = _build(kind, k, dev, rank, world, dist.group.WORLD, collective)
            outs = _run(m, dev)
            if collective == "nvls":
                parallel.nvls_reducer(dist.group.WORLD, 8, dev).check()
            if rank == 0:
                torch.save(outs, os.path.join(out_dir, "tp.pt"))
        dist.barrier()
    finally:
        parallel._REDUCERS.clear()
        torch.cuda.synchronize()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("collective", ["nccl", "nvls"])
@pytest.mark.parametrize("kind,k", [("hcm", 128), ("hcl", 16)])
def test_tp2_matches_single_gpu(kind, k, collective, tmp_path):
    ref = _run(_build(kind, k, torch.device("cuda", 0)), torch.device("cuda", 0))
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, kind, k, port, str(tmp_path), collective))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    got = torch.load(tmp_path / "tp.pt")
    if isinstance(got, str):
        pytest.skip("these GPUs have no NVLink multicast")
    for i, (a, b) in enumerate(zip(got, ref)):
        assert max_rel_err(a, b) < REL_TOL, i
