"""Device-side failure detection on the B200, tested without a GPU fault.

Every pipeline wait inside the kernels is bounded.  Here a test shortens the
limit to 1 ms and makes the attention kernel withhold one barrier arrive (the
first "P ready" of each CTA; no TMA transfer depends on it): the MMA warp's
wait runs out, the CTA records the wait site in the device status word, the
other warps see the abort flag and leave, in-flight copies and MMAs drain,
TMEM is freed and the kernel returns.  The entry point then reports
TJ_ERR_DEVICE (sync check on), the status word is cleared, and the same
context runs the next launch correctly.  A row table in device memory that
points outside its buffer is refused by the kernel itself (kDevBadArgument)
before it touches memory.
"""
from __future__ import annotations

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _case(seed=3):
    g = torch.Generator().manual_seed(seed)
    lengths = [300, 128, 700, 1]
    H = 4
    lens = torch.tensor(lengths, dtype=torch.int32)
    cu = torch.zeros(len(lengths) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    rows = int(cu[-1])
    qkv = torch.randn(3, H, rows, 64, generator=g).half().to(DEV)
    return qkv, cu, lens, max(lengths)


def _reference(qkv, cu, lens):
    q, k, v = (t.float() for t in qkv)
    H = q.shape[0]
    out = torch.zeros(q.shape[1], H * 64, device=q.device)
    for b in range(lens.numel()):
        a, e = int(cu[b]), int(cu[b + 1])
        p = torch.softmax(q[:, a:e] @ k[:, a:e].transpose(1, 2) * 0.125, -1)
        out[a:e] = (p @ v[:, a:e]).transpose(0, 1).reshape(e - a, H * 64)
    return out


def _attention(k, qkv, cu, lens, max_q, q_cu=None):
    q_cu = cu if q_cu is None else q_cu
    return k.flash_attn_fwd(qkv[0], qkv[1:2], qkv[2:3], q_cu.to(DEV), cu[:-1].view(-1, 1).contiguous().to(DEV),
                            lens.view(-1, 1).contiguous().to(DEV), max_q, 0.125)


@pytest.fixture
def debug_knobs(cuda_pkg):
    lib = cuda_pkg._lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    assert cuda_pkg._lib.device_status(stream) == [0, 0, 0, 0]
    prev = cuda_pkg._lib.set_sync_check(True)
    yield lib
    lib.tj_debug_withhold_arrive(cuda_pkg._lib.TJ_WITHHOLD_NONE)
    lib.tj_debug_set_wait_limit_ns(0)
    cuda_pkg._lib.set_sync_check(prev)


def test_withheld_arrive_runs_out_and_kernel_returns(cuda_pkg, debug_knobs):
    lib, L = debug_knobs, cuda_pkg._lib
    k = cuda_pkg.kernels
    qkv, cu, lens, max_q = _case()
    L.check(lib.tj_debug_set_wait_limit_ns(1_000_000), "debug_set_wait_limit_ns")  # 1 ms
    L.check(lib.tj_debug_withhold_arrive(L.TJ_WITHHOLD_ATTN_P_READY), "debug_withhold_arrive")
    t0 = time.perf_counter()
    with pytest.raises(L.TJError) as err:
        _attention(k, qkv, cu, lens, max_q)
    elapsed = time.perf_counter() - t0
    assert err.value.code == L.TJ_ERR_DEVICE
    msg = str(err.value)
    # The withheld arrive stalls the whole pipeline, so whichever bounded wait
    # of the attention kernel started first runs out first: the MMA warp's wait
    # for it (213), the producer's wait for a free K/V stage (200-202) or a
    # softmax warp's (220-223); the others then see the abort flag.
    assert "device error 1" in msg and "time limit" in msg, msg
    assert any(f"site {s}," in msg for s in range(200, 224)), msg
    assert elapsed < 1.0, f"the kernel took {elapsed:.2f} s to give up"
    L.check(lib.tj_debug_withhold_arrive(L.TJ_WITHHOLD_NONE), "debug_withhold_arrive")
    L.check(lib.tj_debug_set_wait_limit_ns(0), "debug_set_wait_limit_ns")
    # the status word was read and cleared; the context is still usable
    assert L.device_status(torch.cuda.current_stream().cuda_stream) == [0, 0, 0, 0]
    out = _attention(k, qkv, cu, lens, max_q)
    assert float((out.float() - _reference(qkv, cu, lens)).abs().max()) < 4e-3


def test_withheld_arrive_inside_the_encoder_reports_a_device_error(cuda_pkg, debug_knobs):
    import oracle

    lib, L = debug_knobs, cuda_pkg._lib
    cfg = oracle.TransformerConfig(2, 256, 256, 4, 1024, 1, False)
    sd = oracle.make_state_dict(cfg, seed=12)
    x, mask = oracle.generate_random_case(cfg, seed=12, padding_ratio=0.5)
    model = cuda_pkg.UserOptimizedTransformer(cuda_pkg.TransformerConfig(*cfg.__dict__.values()))
    model.load_state_dict(sd, strict=True)
    model = model.to(DEV).eval()
    xd, md = x.to(DEV), mask.to(DEV)
    L.check(lib.tj_debug_set_wait_limit_ns(1_000_000), "debug_set_wait_limit_ns")
    L.check(lib.tj_debug_withhold_arrive(L.TJ_WITHHOLD_ATTN_P_READY), "debug_withhold_arrive")
    with torch.inference_mode(), pytest.raises(L.TJError) as err:
        model(xd, md)
    assert err.value.code == L.TJ_ERR_DEVICE and "time limit" in str(err.value), str(err.value)
    L.check(lib.tj_debug_withhold_arrive(L.TJ_WITHHOLD_NONE), "debug_withhold_arrive")
    L.check(lib.tj_debug_set_wait_limit_ns(0), "debug_set_wait_limit_ns")
    with torch.inference_mode():
        out = model(xd, md)
    torch.cuda.synchronize()
    r = oracle.compare_outputs(oracle.encoder_forward(sd, cfg, x, mask), out.cpu())
    assert r.passed, r


def test_row_table_outside_its_buffer_is_refused_by_the_kernel(cuda_pkg, debug_knobs):
    """q_cu's last entry points 100 rows past the query slab: the kernel's own
    check refuses the sample before any load or store."""
    L = cuda_pkg._lib
    k = cuda_pkg.kernels
    qkv, cu, lens, max_q = _case(5)
    bad = cu.clone()
    bad[-1] = int(cu[-1]) + 100
    with pytest.raises(L.TJError) as err:
        _attention(k, qkv, cu, lens, max_q + 100, q_cu=bad)
    msg = str(err.value)
    assert err.value.code == L.TJ_ERR_DEVICE and "device error 2" in msg and "site 230" in msg, msg
    assert L.device_status(torch.cuda.current_stream().cuda_stream) == [0, 0, 0, 0]
    out = _attention(k, qkv, cu, lens, max_q)
    assert float((out.float() - _reference(qkv, cu, lens)).abs().max()) < 4e-3
