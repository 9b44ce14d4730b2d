"""t2sx_matmul_noalloc: the matmul entry point for callers that cannot allocate device memory
at call time (a synthesis thread that must not let cudaMalloc synchronise the device, or a host
application that owns the whole device memory budget).  It must give exactly the result of
t2sx_matmul -- this suite's tolerance for matmuls is bit equality -- on consecutive calls that
share its fixed scratch array, and reject sizes beyond that array with a clear error.

Kept in a file that pytest collects last, so a run stopping at its first failure has already
run every other test; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _weight_bytes(fmt, N, K, seed):
    import gguf
    import synth
    w = (np.random.default_rng(seed).standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    if fmt == "q8_0":
        return 8, gguf.quantize(w, gguf.GGMLQuantizationType.Q8_0)
    if fmt == "q4_k":
        return 12, synth.quantize_q4_k(w)
    return 1, w.astype(np.float16).view(np.uint8)


def _weight(t2sx_mod, fmt, N, K, seed):
    wt, wb = _weight_bytes(fmt, N, K, seed)
    return t2sx_mod.Weight(wt, wb, N, K)


def _both(w, x, N, bias=None):
    M = x.shape[0]
    xd = torch.from_numpy(x).cuda()
    bd = None if bias is None else torch.from_numpy(bias).cuda()
    y_ref = torch.empty((M, N), dtype=torch.float32, device="cuda")
    y_new = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    w.matmul(xd.data_ptr(), M, y_ref.data_ptr(), None if bd is None else bd.data_ptr(), stream=stream)
    w.matmul_noalloc(xd.data_ptr(), M, y_new.data_ptr(), None if bd is None else bd.data_ptr(), stream=stream)
    torch.cuda.synchronize()
    return y_ref.cpu().numpy(), y_new.cpu().numpy()


def test_noalloc_matches_matmul_on_consecutive_calls(t2sx_mod):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required")
    rng = np.random.default_rng(0)
    # q4_k at M = 4096, K = 512 (the tcgen05 path, its TMA map over the fixed array) and q8_0 at
    # M = 1024, K = 2048 fill the array exactly: M * K == NOALLOC_MAX_ELEMS
    cases = [("q8_0", 1536, 512, 64), ("q4_k", 512, 2048, 40), ("f16", 1025, 512, 5), ("q8_0", 512, 512, 1),
             ("q4_k", 1536, 512, 96), ("q4_k", 512, 512, 4096), ("q8_0", 512, 2048, 1024)]
    assert 512 * 4096 == t2sx_mod.NOALLOC_MAX_ELEMS and 2048 * 1024 == t2sx_mod.NOALLOC_MAX_ELEMS
    for i, (fmt, N, K, M) in enumerate(cases):
        w = _weight(t2sx_mod, fmt, N, K, seed=i)
        x = rng.standard_normal((M, K), dtype=np.float32)
        bias = rng.standard_normal(N, dtype=np.float32) if i % 2 == 0 else None
        ref, new = _both(w, x, N, bias)
        assert np.array_equal(ref.view(np.uint32), new.view(np.uint32)), (fmt, N, K, M)
        # a second call on the same scratch with different data
        x2 = rng.standard_normal((M, K), dtype=np.float32) * 3
        ref2, new2 = _both(w, x2, N, bias)
        assert np.array_equal(ref2.view(np.uint32), new2.view(np.uint32)), (fmt, N, K, M, "second call")
        w.close()


def test_noalloc_rejects_oversized_inputs(t2sx_mod):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required")
    K = 2048
    w = _weight(t2sx_mod, "q8_0", 512, K, seed=9)
    M = t2sx_mod.NOALLOC_MAX_ELEMS // K + 1
    x = torch.zeros((M, K), dtype=torch.float32, device="cuda")
    y = torch.zeros((M, 512), dtype=torch.float32, device="cuda")
    with pytest.raises(t2sx_mod.T2SXError) as e:
        w.matmul_noalloc(x.data_ptr(), M, y.data_ptr())
    assert e.value.code == t2sx_mod.ERR_INVALID and "exceed the fixed scratch" in str(e.value)
    # a row count whose product with K overflows 64 bits is refused the same way
    with pytest.raises(t2sx_mod.T2SXError) as e:
        w.matmul_noalloc(x.data_ptr(), 1 << 62, y.data_ptr())
    assert e.value.code == t2sx_mod.ERR_INVALID
    w.close()


def test_noalloc_matches_oracle(t2sx_mod, orc):
    """The no-allocation matmul against the CPU oracle (bit for bit, bias added after the dot as
    the layer does), at sizes that fill the fixed array and on the tcgen05 path."""
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required")
    rng = np.random.default_rng(5)
    for i, (fmt, N, K, M) in enumerate([("q4_k", 512, 512, 4096), ("q8_0", 512, 2048, 1024), ("q4_k", 1536, 512, 200),
                                        ("f16", 1025, 512, 3)]):
        wt, wb = _weight_bytes(fmt, N, K, seed=100 + i)
        w = t2sx_mod.Weight(wt, wb, N, K)
        x = rng.standard_normal((M, K), dtype=np.float32)
        bias = rng.standard_normal(N, dtype=np.float32)
        ref = orc.matmul(wt, wb.reshape(-1), N, K, x) + bias[None, :]
        xd = torch.from_numpy(x).cuda()
        bd = torch.from_numpy(bias).cuda()
        for call in range(2):   # two calls in a row share the array
            y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
            w.matmul_noalloc(xd.data_ptr(), M, y.data_ptr(), bd.data_ptr(),
                             stream=torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            got = y.cpu().numpy()
            assert np.array_equal(got.view(np.uint32), ref.astype(np.float32).view(np.uint32)), (fmt, N, K, M, call)
        w.close()
