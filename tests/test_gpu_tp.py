"""Tensor-parallel decode over NVLink (configs[4] mode b) on 2 GPUs.

Two spawned ranks, one per GPU, exchange CUDA IPC handles over NCCL's
host-side object gather and then decode with the MLP and LM-head rows split;
the kernels exchange partial sums and argmax pairs over NVLink.  Checked on
rank 0 against the golden vectors of the reference's fp32 forward, with the
same gates as the single-GPU parity tests, for agreement between ranks, and
against NCCL: the partial sums that arrived over NVLink equal the ones NCCL
gathers, their sum NCCL's all_reduce, and the in-kernel argmax the argmax of
the logits NCCL gathers.
Skipped on a box with fewer than 2 GPUs.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from ._common import LOGIT_TOL, MARGIN, golden, weights

pytestmark = pytest.mark.gpu
WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from megakernel_b200 import tp
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    res = {}
    for name in ["tiny", "qwen3-0.6b-d64"]:
        shape, _, flat, offs = weights(name)
        g = golden(name)
        eng = tp.make_engine(flat, offs, shape, device=rank, max_seq=1024, timeout_ns=2_000_000_000)
        seq = g["seq"].tolist()
        n = len(seq)
        toks = torch.tensor(seq, dtype=torch.int32, device=dev)
        o = torch.zeros(n, dtype=torch.int32, device=dev)
        lg = torch.zeros(n, shape.vocab, dtype=torch.float32, device=dev)
        eng.decode_n(toks, n, o, logits=lg)
        full = tp.gather_logits(lg, shape.vocab).cpu().numpy()
        # Cross-check of the in-kernel NVLink exchange with NCCL: the partial
        # down projections of the last layer as they arrived in this GPU's
        # exchange slots equal every rank's own partial gathered by NCCL, and
        # their rank-order sum equals NCCL's all_reduce of the partials.
        slots = torch.zeros(world, shape.hidden, dtype=torch.float32, device=dev)
        assert eng.lib.megakernel_tp_exchange_slots(eng._handle, slots.data_ptr()) == 0
        own = slots[rank].clone()
        gathered = [torch.zeros_like(own) for _ in range(world)]
        dist.all_gather(gathered, own)
        red = own.clone()
        dist.all_reduce(red)
        slots_equal_nccl = all(bool(torch.equal(slots[j], gathered[j])) for j in range(world))
        ssum = slots[0].clone()
        for j in range(1, world):
            ssum += slots[j]
        sum_err = float((ssum - red).abs().max() / red.abs().max().clamp_min(1e-30))
        allo = [torch.zeros_like(o) for _ in range(world)]
        dist.all_gather(allo, o)
        # free-running greedy from the prompt
        eng.reset()
        n_prompt = int(g["n_prompt"])
        fr = torch.zeros(n - 1, dtype=torch.int32, device=dev)
        eng.decode_n(toks[:n_prompt].contiguous(), n_prompt, fr, n_steps=n - 1)
        if rank == 0:
            from megakernel_b200.bridge import MegakernelEngine
            e1 = MegakernelEngine(flat=flat, offsets=offs, shape=shape, device=rank, max_seq=1024)
            fr1 = torch.zeros(n - 1, dtype=torch.int32, device=dev)
            e1.decode_n(toks[:n_prompt].contiguous(), n_prompt, fr1, n_steps=n - 1)
            e1.close()
            err_sub = float(np.abs(full[:, g["sub_ids"]] - g["sub_logits"]).max())
            top = np.take_along_axis(full, g["top_ids"], axis=1)
            err_top = float(np.abs(top - g["top_vals"]).max())
            ok = g["margin"] > MARGIN
            got = fr.cpu().numpy()[n_prompt - 1:]
            want = g["seq"][n_prompt:]
            low = np.nonzero(g["margin"][n_prompt - 1:-1] <= MARGIN)[0]
            upto = int(low[0]) if low.size else len(want)
            res[name] = dict(
                err=max(err_sub, err_top),
                argmax_ok=bool(np.array_equal(o.cpu().numpy()[ok], g["argmax"][ok])),
                full_argmax_ok=bool(np.array_equal(full.argmax(1), o.cpu().numpy())),
                ranks_agree=all(bool(torch.equal(a, allo[0])) for a in allo),
                greedy_ok=bool(np.array_equal(got[:upto], want[:upto])),
                tp_equals_single_gpu=bool(torch.equal(fr, fr1)),
                slots_equal_nccl=slots_equal_nccl, slot_sum_vs_allreduce=sum_err)
        eng.close()
    if rank == 0:
        out.update(res)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_tensor_parallel_vs_reference_2gpu():
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(WORLD, _free_port(), out), nprocs=WORLD, join=True)
    for name in ["tiny", "qwen3-0.6b-d64"]:
        r = out[name]
        assert r["err"] < LOGIT_TOL, (name, r)
        assert r["argmax_ok"] and r["full_argmax_ok"] and r["ranks_agree"], (name, r)
        assert r["greedy_ok"] and r["tp_equals_single_gpu"], (name, r)
        assert r["slots_equal_nccl"] and r["slot_sum_vs_allreduce"] < 1e-6, (name, r)
