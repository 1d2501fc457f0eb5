"""tcgen05 GEMM of the batched path (megakernel_tc_gemm_test) against torch.

x fp32 [rows x K] enters the tensor cores as bf16 hi + lo terms, W is bf16;
the result must match x @ W^T computed in fp64 to 2e-5 of the output's
largest magnitude (the lo term leaves ~2^-17 of x unrepresented;
accumulation is fp32).
"""
import ctypes

import pytest
import torch

from megakernel_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("rows,K,N", [(64, 1024, 2048), (64, 2816, 1024), (7, 1024, 5632), (64, 64, 64), (64, 4096, 128)])
def test_tc_gemm_matches_fp64(rows, K, N):
    L = _lib.load()
    g = torch.Generator(device="cpu").manual_seed(rows * 7 + K + N)
    x = torch.randn(rows, K, generator=g).to(DEV)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    out = torch.zeros(rows, N, device=DEV)
    rc = L.megakernel_tc_gemm_test(ctypes.c_void_p(x.data_ptr()), rows, ctypes.c_void_p(w.data_ptr()), K, N,
                                   ctypes.c_void_p(out.data_ptr()), None)
    assert rc == 0, rc
    ref = x.double() @ w.double().t()
    err = ((out.double() - ref).abs().max() / ref.abs().max()).item()
    assert err < 2e-5, err


@pytest.mark.parametrize("rows,K,N", [(64, 1024, 2048), (64, 2816, 1024), (5, 1024, 256)])
def test_tc_gemm_e4m3_weights_match_fp64(rows, K, N):
    """The e4m3-weight form (converter warps expand each W block to bf16 in
    shared memory; per-row scales in the epilogue) against x @ (s * q)^T in
    fp64 with the same e4m3 values."""
    L = _lib.load()
    g = torch.Generator(device="cpu").manual_seed(rows + K + 3 * N)
    x = torch.randn(rows, K, generator=g).to(DEV)
    w = torch.randn(N, K, generator=g) * 0.02
    sc = w.abs().amax(dim=1) / 448.0
    q = (w / sc[:, None]).to(torch.float8_e4m3fn)
    q_dev, sc_dev = q.view(torch.uint8).to(DEV), sc.to(DEV)
    out = torch.zeros(rows, N, device=DEV)
    rc = L.megakernel_tc_gemm_test_e4m3(ctypes.c_void_p(x.data_ptr()), rows, ctypes.c_void_p(q_dev.data_ptr()),
                                        ctypes.c_void_p(sc_dev.data_ptr()), K, N, ctypes.c_void_p(out.data_ptr()),
                                        None)
    assert rc == 0, rc
    ref = x.double() @ (q.double() * sc.double()[:, None]).t().to(DEV)
    err = ((out.double() - ref).abs().max() / ref.abs().max()).item()
    assert err < 2e-5, err


@pytest.mark.parametrize("rows,K,N,ksplit", [(64, 2816, 1024, 3), (64, 2816, 1024, 4), (64, 1024, 1024, 4),
                                             (64, 1024, 5632, 2), (64, 1024, 5632, 4), (9, 1024, 2048, 4),
                                             (64, 128, 64, 2)])
def test_tc_gemm_split_k_cluster(rows, K, N, ksplit):
    """K split over a cluster of `ksplit` CTAs per tile, partials pushed into
    rank 0's shared memory and summed there: matches fp64 like the unsplit
    GEMM, and is deterministic (two runs equal bit for bit).  N = 5632 has
    more tiles than fit one wave of clusters, so CTAs loop over tiles and
    reuse the receive buffers."""
    L = _lib.load()
    g = torch.Generator(device="cpu").manual_seed(rows * 11 + K + N + ksplit)
    x = torch.randn(rows, K, generator=g).to(DEV)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    outs = []
    for _ in range(2):
        out = torch.zeros(rows, N, device=DEV)
        rc = L.megakernel_tc_gemm_test_split(ctypes.c_void_p(x.data_ptr()), rows, ctypes.c_void_p(w.data_ptr()), K,
                                             N, ksplit, ctypes.c_void_p(out.data_ptr()), None)
        assert rc == 0, rc
        outs.append(out)
    ref = x.double() @ w.double().t()
    err = ((outs[0].double() - ref).abs().max() / ref.abs().max()).item()
    assert err < 2e-5, err
    assert torch.equal(outs[0], outs[1])
