"""Per-kernel parity on the B200, through the C ABI (kernels.py -> ctypes).

Each kernel is compared with a plain PyTorch FP32 (or float64) computation of
the same op on the same fp16 operands; tolerances are written per test.
"""
from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(autouse=True)
def _sync_check(cuda_pkg):
    prev = cuda_pkg._lib.set_sync_check(True)
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    cuda_pkg._lib.set_sync_check(prev)


def _plan_reference(mask):
    B, S = mask.shape
    flat = mask.reshape(-1).bool()
    orig = torch.nonzero(flat).flatten().int()
    inv = torch.full((B * S,), -1, dtype=torch.int32)
    inv[orig.long()] = torch.arange(orig.numel(), dtype=torch.int32)
    counts = mask.sum(1).int()
    cu = torch.zeros(B + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(counts, 0)
    return orig, inv, counts, cu


# The plan runs one CTA per >= 4096 mask bytes (at most 256 CTAs): samples
# cross CTA segments (5x3001, 1x131072), many start inside one (20000x1,
# 300x129: above 256 samples the order is the identity), 3x1000003 spreads
# over 256 CTAs, and a mask that starts off a 16-byte boundary takes the
# byte-load path.
@pytest.mark.parametrize("B,S,offset", [(1, 1, 0), (2, 8, 0), (40, 7, 0), (33, 33, 0), (3, 1000, 0),
                                        (8, 2048, 0), (1, 131072, 0), (5, 3001, 0), (20000, 1, 0),
                                        (300, 129, 0), (3, 1000003, 0), (8, 2048, 1), (5, 3001, 3)])
def test_token_plan(cuda_pkg, B, S, offset):
    k = cuda_pkg.kernels
    g = torch.Generator().manual_seed(B * 7 + S)
    lengths = torch.randint(0, S + 1, (B,), generator=g)
    mask = torch.arange(S)[None, :] < lengths[:, None]
    if B >= 3:
        mask[1] = torch.rand(S, generator=g) < 0.3  # a non-prefix row
        mask[0] = False  # an all-padded row
    store = torch.zeros(B * S + offset, dtype=torch.bool, device=DEV)
    dmask = store[offset:].view(B, S)
    dmask.copy_(mask.to(DEV))
    plan = k.token_plan(dmask, B, S, DEV)
    nv, cu, cnt, orig, inv = [t.cpu() for t in k.plan_views(plan, B, S)]
    r_orig, r_inv, r_cnt, r_cu = _plan_reference(mask)
    assert int(nv) == int(mask.sum())
    assert torch.equal(cu, r_cu)
    assert torch.equal(cnt, r_cnt)
    assert torch.equal(orig[: int(nv)], r_orig)
    assert torch.equal(inv, r_inv)
    order = k.plan_order(plan, B, S).cpu()
    if B <= 256:  # longest first, ties by sample index
        ref_order = sorted(range(B), key=lambda b: (-int(r_cnt[b]), b))
        assert order.tolist() == ref_order
    else:
        assert torch.equal(order, torch.arange(B, dtype=torch.int32))
    # No mask: identity plan.
    plan = k.token_plan(None, B, S, DEV)
    nv, cu, cnt, orig, inv = [t.cpu() for t in k.plan_views(plan, B, S)]
    assert int(nv) == B * S
    assert torch.equal(orig, torch.arange(B * S, dtype=torch.int32))
    assert torch.equal(cnt, torch.full((B,), S, dtype=torch.int32))
    assert torch.equal(cu, torch.arange(B + 1, dtype=torch.int32) * S)


# D above 4096 runs a CTA per row (4100: 8 groups per thread, the last partly
# used; 12288: 16; 32768: 32, the widest row).
@pytest.mark.parametrize("rows,D", [(5, 16), (300, 256), (1000, 768), (513, 1024), (64, 4096),
                                    (40, 4100), (33, 8192), (20, 12288), (9, 32768),
                                    # D % 4 != 0: one column per group
                                    (7, 30), (50, 1001), (3, 5001)])
def test_ln_cast_and_final(cuda_pkg, rows, D):
    k = cuda_pkg.kernels
    g = torch.Generator().manual_seed(rows + D)
    x = torch.randn(rows, D, generator=g) * 3 + 0.5
    gamma = 1 + 0.1 * torch.randn(D, generator=g)
    beta = 0.1 * torch.randn(D, generator=g)
    ref = torch.nn.functional.layer_norm(x.double(), (D,), gamma.double(), beta.double(), 1e-5)
    xd, gd, bd = x.to(DEV), gamma.to(DEV), beta.to(DEV)
    y16 = k.ln_cast_f16(xd, gd, bd).cpu().double()
    # fp16 rounding of the fp32 result: <= 1 ulp of fp16 (2^-10 relative) plus fp32 noise.
    assert torch.all((y16 - ref).abs() <= ref.abs() * 2**-10 + 1e-5)
    # gather map + row count
    perm = torch.randperm(rows, generator=g).int()
    cnt = torch.tensor([rows // 2], dtype=torch.int32)
    y16m = k.ln_cast_f16(xd, gd, bd, row_map=perm.to(DEV), row_count=cnt.to(DEV)).cpu().double()
    half = rows // 2
    refm = ref[perm.long()[:half]]
    assert torch.all((y16m[:half] - refm).abs() <= refm.abs() * 2**-10 + 1e-5)
    # final LN with inverse map and padded rows
    inv = torch.arange(rows, dtype=torch.int32)
    inv[::3] = -1
    out = k.ln_final_mask(xd, gd, bd, inv_map=inv.to(DEV)).cpu().double()
    valid = inv >= 0
    torch.testing.assert_close(out[valid], ref[valid], rtol=0, atol=2e-5)
    assert torch.count_nonzero(out[~valid]) == 0


def test_ln_rejects_rows_above_32768(cuda_pkg):
    k = cuda_pkg.kernels
    D = 32772
    x = torch.zeros(2, D, device=DEV)
    gamma, beta = torch.ones(D, device=DEV), torch.zeros(D, device=DEV)
    with pytest.raises(RuntimeError, match="above 32768"):
        k.ln_cast_f16(x, gamma, beta)
    with pytest.raises(RuntimeError, match="above 32768"):
        k.ln_final_mask(x, gamma, beta)


@pytest.mark.parametrize("rows,D", [(5, 16), (300, 256), (513, 1024), (64, 4096), (17, 8192),
                                    (9, 32768), (9, 30), (5, 5001)])
def test_add_ln_cast_and_final(cuda_pkg, rows, D):
    """Residual add (fp32 x + fp16 branch output) fused into the LayerNorm."""
    k = cuda_pkg.kernels
    g = torch.Generator().manual_seed(rows * 3 + D)
    x = torch.randn(rows + 5, D, generator=g) * 3 + 0.5
    add = (torch.randn(rows, D, generator=g) * 2).half()
    gamma = 1 + 0.1 * torch.randn(D, generator=g)
    beta = 0.1 * torch.randn(D, generator=g)
    perm = torch.randperm(rows + 5, generator=g)[:rows].int()
    cnt = rows - rows // 4
    s_ref = x[perm.long()] + add.float()  # fp32, the reference's `x + out.float()`
    ref = torch.nn.functional.layer_norm(s_ref.double(), (D,), gamma.double(), beta.double(), 1e-5)
    xd, ad, gd, bd = x.to(DEV), add.to(DEV), gamma.to(DEV), beta.to(DEV)
    sum_out = torch.full((rows, D), float("nan"), device=DEV)
    y16 = k.add_ln_cast_f16(xd, ad, gd, bd, row_map=perm.to(DEV),
                            row_count=torch.tensor([cnt], dtype=torch.int32, device=DEV),
                            sum_out=sum_out).cpu().double()
    assert torch.equal(sum_out[:cnt].cpu(), s_ref[:cnt]), "fp32 residual sum must be exact"
    assert torch.isnan(sum_out[cnt:].cpu()).all(), "rows past the count must not be written"
    assert torch.all((y16[:cnt] - ref[:cnt]).abs() <= ref[:cnt].abs() * 2**-10 + 1e-5)
    # final LN of x + add, scattered through an inverse map with padded rows
    xc = x[:rows].contiguous()
    s2 = xc + add.float()
    ref2 = torch.nn.functional.layer_norm(s2.double(), (D,), gamma.double(), beta.double(), 1e-5)
    inv = torch.full((rows + 7,), -1, dtype=torch.int32)
    slots = torch.randperm(rows + 7, generator=g)[:rows]
    inv[slots] = torch.arange(rows, dtype=torch.int32)
    out = k.add_ln_final_mask(xc.to(DEV), ad, gd, bd, inv_map=inv.to(DEV)).cpu().double()
    torch.testing.assert_close(out[slots], ref2, rtol=0, atol=2e-5)
    assert torch.count_nonzero(out[inv < 0]) == 0


@pytest.mark.parametrize("x_at_original", [True, False])
@pytest.mark.parametrize("D", [1024, 6144])
def test_add2_ln_final(cuda_pkg, x_at_original, D):
    """The last layer's two residual adds fused with the final LayerNorm and the
    scatter: LN((x + attn) + ffn), x read at the output row or the compact row."""
    k = cuda_pkg.kernels
    g = torch.Generator().manual_seed(3 + int(x_at_original) + D)
    rows = 700
    inv = torch.full((rows,), -1, dtype=torch.int32)
    valid = torch.randperm(rows, generator=g)[:500].sort().values
    inv[valid] = torch.arange(500, dtype=torch.int32)
    nvr = 500
    attn = (torch.randn(nvr, D, generator=g) * 2).half()
    ffn = (torch.randn(nvr, D, generator=g) * 2).half()
    gamma = 1 + 0.1 * torch.randn(D, generator=g)
    beta = 0.1 * torch.randn(D, generator=g)
    if x_at_original:
        x = torch.randn(rows, D, generator=g) * 3
        xs = x[valid]
    else:
        x = torch.randn(nvr, D, generator=g) * 3
        xs = x
    s_ref = (xs + attn.float()) + ffn.float()
    ref = torch.nn.functional.layer_norm(s_ref.double(), (D,), gamma.double(), beta.double(), 1e-5)
    out = k.add2_ln_final_mask(x.to(DEV), attn.to(DEV), ffn.to(DEV), gamma.to(DEV), beta.to(DEV),
                               inv_map=inv.to(DEV), x_at_original=x_at_original, rows=rows).cpu().double()
    torch.testing.assert_close(out[valid], ref, rtol=0, atol=2e-5)
    assert torch.count_nonzero(out[inv < 0]) == 0


def _gemm_ref(a16, w16, bias):
    return a16.float() @ w16.float().t() + bias


@pytest.mark.parametrize(
    "rows,count,D,H",
    [(128, 128, 256, 4), (1000, 777, 768, 12), (4096, 4096, 1024, 16), (300, 0, 256, 4),
     (200, 150, 256, 8), (40, 33, 16, 4), (77, 77, 96, 4),
     # CTA-pair tiles (256 rows): second CTA partly valid / without valid rows / past rows_max
     (5000, 4321, 768, 12), (5000, 4196, 768, 12), (4100, 4100, 768, 12),
     # head dims above 64: rows padded to 128 / 256 halves
     (500, 480, 256, 2), (300, 300, 512, 2), (200, 190, 192, 2), (100, 100, 320, 2), (64, 64, 144, 2)],
)
def test_gemm_qkv_headmajor(cuda_pkg, rows, count, D, H):
    """Head-major output [3][H][rows][P]; head dims below P (64/128/256) zero-padded."""
    k = cuda_pkg.kernels
    dh = D // H
    P = k.head_pad(dh)
    g = torch.Generator().manual_seed(rows + D)
    a = torch.randn(rows, D, generator=g).half().to(DEV)
    w = (torch.randn(3 * D, D, generator=g) / math.sqrt(D)).half().to(DEV)
    b = torch.randn(3 * D, generator=g).to(DEV)
    out = torch.full((3, H, rows, P), float("nan"), dtype=torch.float16, device=DEV)
    k.gemm_qkv_headmajor(a, w, b, H, row_count=torch.tensor([count], dtype=torch.int32, device=DEV), out=out)
    ref = _gemm_ref(a, w, b)  # [rows, 3D]
    ref_hm = ref.view(rows, 3, H, dh).permute(1, 2, 0, 3)
    got = out[:, :, :count, :dh].float()
    exp = ref_hm[:, :, :count]
    # fp32 accumulation of fp16 products, then one fp16 rounding.
    assert torch.all((got - exp).abs() <= exp.abs() * 2**-10 + 2e-3), float((got - exp).abs().max())
    if dh < P:
        assert torch.count_nonzero(out[:, :, :count, dh:].float()) == 0, "head padding must be zero"
    if count < rows:
        assert torch.isnan(out[:, :, count:].float()).all(), "rows past the count must not be written"


@pytest.mark.parametrize("rows,count,N,K",
                         [(256, 200, 1024, 1024), (1000, 1000, 768, 3072), (640, 513, 256, 256), (40000, 39000, 1024, 1024),
                          (30000, 29999, 640, 512)])
def test_gemm_bias_residual_f32(cuda_pkg, rows, count, N, K):
    k = cuda_pkg.kernels
    g = torch.Generator().manual_seed(rows + N + K)
    a = torch.randn(rows, K, generator=g).half().to(DEV)
    w = (torch.randn(N, K, generator=g) / math.sqrt(K)).half().to(DEV)
    b = torch.randn(N, generator=g).to(DEV)
    resid = torch.randn(rows + 7, N, generator=g).to(DEV)
    rmap = torch.randperm(rows + 7, generator=g)[:rows].int().to(DEV)
    out = k.gemm_bias_residual_f32(a, w, b, resid, resid_map=rmap,
                                   row_count=torch.tensor([count], dtype=torch.int32, device=DEV))
    ref = _gemm_ref(a, w, b) + resid[rmap.long()]
    torch.testing.assert_close(out[:count], ref[:count], rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("rows,N,K", [(512, 4096, 1024), (333, 3072, 768), (128, 1024, 256), (100, 136, 96),
                                      (9000, 4096, 1024), (12000, 1000, 512)])
def test_gemm_bias_gelu_f16(cuda_pkg, rows, N, K):
    k = cuda_pkg.kernels
    g = torch.Generator().manual_seed(rows + N)
    a = torch.randn(rows, K, generator=g).half().to(DEV)
    w = (torch.randn(N, K, generator=g) / math.sqrt(K)).half().to(DEV)
    b = torch.randn(N, generator=g).to(DEV)
    out = k.gemm_bias_gelu_f16(a, w, b).float()
    ref = torch.nn.functional.gelu(_gemm_ref(a, w, b), approximate="none")
    assert torch.all((out - ref).abs() <= ref.abs() * 2**-10 + 2e-3), float((out - ref).abs().max())


@pytest.mark.parametrize("rows,count,N,K", [(300, 300, 1024, 1024), (1000, 777, 136, 96),
                                           (12416, 12000, 1024, 1024), (9000, 9000, 1000, 4096)])
def test_gemm_bias_f16(cuda_pkg, rows, count, N, K):
    k = cuda_pkg.kernels
    g = torch.Generator().manual_seed(rows + N + K + 1)
    a = torch.randn(rows, K, generator=g).half().to(DEV)
    w = (torch.randn(N, K, generator=g) / math.sqrt(K)).half().to(DEV)
    b = torch.randn(N, generator=g).to(DEV)
    out = torch.full((rows, N), float("nan"), dtype=torch.float16, device=DEV)
    k.gemm_bias_f16(a, w, b, row_count=torch.tensor([count], dtype=torch.int32, device=DEV), out=out)
    ref = _gemm_ref(a, w, b)[:count]
    got = out[:count].float()
    assert torch.all((got - ref).abs() <= ref.abs() * 2**-10 + 2e-3), float((got - ref).abs().max())
    if count < rows:
        assert torch.isnan(out[count:].float()).all(), "rows past the count must not be written"


def _attn_ref(q, k, v, q_cu, kv_off, kv_len, scale, causal=False, dh=64):
    """q [H, rows, P] fp16; k/v [G, H, rows, P]; fp32 math per sample."""
    H = q.shape[0]
    q, k, v = q[..., :dh], k[..., :dh], v[..., :dh]
    out = torch.zeros(q.shape[1], H * dh, dtype=torch.float32, device=q.device)
    B = q_cu.numel() - 1
    G = k.shape[0]
    for b in range(B):
        q0, q1 = int(q_cu[b]), int(q_cu[b + 1])
        if q1 == q0:
            continue
        ks, vs = [], []
        for gidx in range(G):
            o, l = int(kv_off[b, gidx]), int(kv_len[b, gidx])
            ks.append(k[gidx, :, o : o + l].float())
            vs.append(v[gidx, :, o : o + l].float())
        kk = torch.cat(ks, dim=1)
        vv = torch.cat(vs, dim=1)
        s = torch.matmul(q[:, q0:q1].float(), kk.transpose(-1, -2)) * scale
        if causal:
            qp = torch.arange(q1 - q0, device=q.device)[:, None]
            kp = torch.arange(kk.shape[1], device=q.device)[None, :]
            s = s.masked_fill(kp > qp, float("-inf"))
        p = torch.softmax(s, dim=-1)
        out[q0:q1] = torch.matmul(p, vv).transpose(0, 1).reshape(q1 - q0, H * dh)
    return out


@pytest.mark.parametrize(
    "lengths,H",
    [([1], 1), ([128], 2), ([200, 1, 0, 129], 4), ([1024, 1536, 2048, 700], 16), ([127, 255, 383], 12)],
)
@pytest.mark.parametrize("causal", [False, True])
def test_flash_attention_compact(cuda_pkg, lengths, H, causal):
    k = cuda_pkg.kernels
    g = torch.Generator().manual_seed(sum(lengths) + H)
    lens = torch.tensor(lengths, dtype=torch.int32)
    cu = torch.zeros(len(lengths) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    rows = int(cu[-1]) + 64  # slack rows hold garbage (NaN) that must never leak in
    qkv = torch.randn(3, H, rows, 64, generator=g).half()
    qkv[:, :, int(cu[-1]):] = float("nan")
    qkv = qkv.to(DEV)
    q, kk, vv = qkv[0], qkv[1:2], qkv[2:3]
    kv_off = cu[:-1].view(-1, 1).contiguous()
    kv_len = lens.view(-1, 1).contiguous()
    scale = 64**-0.5
    out = k.flash_attn_fwd(q, kk, vv, cu.to(DEV), kv_off.to(DEV), kv_len.to(DEV), max(lengths), scale,
                           causal=causal)
    ref = _attn_ref(q, kk, vv, cu, kv_off, kv_len, scale, causal)
    n = int(cu[-1])
    err = (out[:n].float() - ref[:n]).abs()
    assert torch.isfinite(out[:n].float()).all()
    assert float(err.max()) < 4e-3, float(err.max())


@pytest.mark.parametrize("pattern", ["growing", "spike"])
@pytest.mark.parametrize("causal", [False, True])
def test_flash_attention_rising_max(cuda_pkg, pattern, causal):
    """Scores whose row max rises by far more than fp16 can absorb across key
    tiles (growing key norms), or jumps by ~100 in one key (a spike): the
    kernel must raise its running max and rescale, whichever way it finds out."""
    k = cuda_pkg.kernels
    g = torch.Generator().manual_seed(5 + causal)
    lengths = [1500, 700, 300]
    H = 2
    lens = torch.tensor(lengths, dtype=torch.int32)
    cu = torch.zeros(len(lengths) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    rows = int(cu[-1])
    qkv = torch.randn(3, H, rows, 64, generator=g)
    for b in range(len(lengths)):
        q0, q1 = int(cu[b]), int(cu[b + 1])
        pos = torch.arange(q1 - q0, dtype=torch.float32)
        if pattern == "growing":
            qkv[1, :, q0:q1] *= (0.2 + 6.0 * pos / (q1 - q0))[None, :, None]
        else:
            qkv[1, :, q0 + (q1 - q0) * 3 // 5] = 40.0
    qkv = qkv.half().to(DEV)
    q, kk, vv = qkv[0], qkv[1:2], qkv[2:3]
    kv_off = cu[:-1].view(-1, 1).contiguous()
    kv_len = lens.view(-1, 1).contiguous()
    scale = 64**-0.5
    out = k.flash_attn_fwd(q, kk, vv, cu.to(DEV), kv_off.to(DEV), kv_len.to(DEV), max(lengths), scale,
                           causal=causal)
    ref = _attn_ref(q, kk, vv, cu, kv_off, kv_len, scale, causal)
    err = (out.float() - ref).abs()
    assert torch.isfinite(out.float()).all()
    assert float(err.max()) < 4e-3, float(err.max())


def test_flash_attention_more_samples_than_grid_rows(cuda_pkg):
    """70000 samples (of 1-3 tokens, and four of 200 tokens placed after grid
    row 65535): more than the 65535 rows of one launch's grid, so the library
    runs it as two launches; the long samples check that the second launch
    finds its samples through its first-row offset."""
    k = cuda_pkg.kernels
    g = torch.Generator().manual_seed(70000)
    B, H = 70000, 1
    lens = torch.randint(1, 4, (B,), generator=g, dtype=torch.int32)
    long_ids = (65535, 65540, 68000, 69999)
    lens[list(long_ids)] = 200
    cu = torch.zeros(B + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    rows = int(cu[-1])
    qkv = torch.randn(3, H, rows, 64, generator=g).half()
    scale = 64**-0.5
    dev = qkv.to(DEV)
    out = k.flash_attn_fwd(dev[0], dev[1:2], dev[2:3], cu.to(DEV), cu[:-1].view(-1, 1).contiguous().to(DEV),
                           lens.view(-1, 1).contiguous().to(DEV), 200, scale).float().cpu()
    # Reference per length group (every sample of length L at once).
    ref = torch.zeros(rows, H * 64)
    q, kk, vv = qkv[0, 0].float(), qkv[1, 0].float(), qkv[2, 0].float()
    for L in (1, 2, 3, 200):
        idx = torch.nonzero(lens == L).flatten()
        rws = (cu[idx].long()[:, None] + torch.arange(L)[None, :])  # [n, L]
        s = torch.einsum("nid,njd->nij", q[rws], kk[rws]) * scale
        ref[rws.reshape(-1)] = torch.einsum("nij,njd->nid", torch.softmax(s, -1), vv[rws]).reshape(-1, 64)
    assert float((out - ref).abs().max()) < 4e-3


def test_flash_attention_segments(cuda_pkg):
    """Two key segments per sample (the context-parallel layout [G][H][rows][64])."""
    k = cuda_pkg.kernels
    g = torch.Generator().manual_seed(11)
    H, G, seg_rows = 4, 2, 512
    q_rows = 300
    q = torch.randn(H, q_rows, 64, generator=g).half().to(DEV)
    kv = torch.randn(G, 2, H, seg_rows, 64, generator=g).half().to(DEV)
    kk, vv = kv[:, 0], kv[:, 1]
    q_cu = torch.tensor([0, q_rows], dtype=torch.int32)
    kv_off = torch.tensor([[0, 0]], dtype=torch.int32)
    kv_len = torch.tensor([[512, 389]], dtype=torch.int32)
    out = k.flash_attn_fwd(q, kk, vv, q_cu.to(DEV), kv_off.to(DEV), kv_len.to(DEV), q_rows, 0.125)
    ref = _attn_ref(q, kk, vv, q_cu, kv_off, kv_len, 0.125)
    assert float((out.float() - ref).abs().max()) < 4e-3


@pytest.mark.parametrize("dh", [4, 8, 32])
def test_flash_attention_small_heads(cuda_pkg, dh):
    """Head dims below 64: rows zero-padded to 64, context holds dh columns per head."""
    k = cuda_pkg.kernels
    g = torch.Generator().manual_seed(dh)
    H = 4
    lens = torch.tensor([300, 77], dtype=torch.int32)
    cu = torch.tensor([0, 300, 377], dtype=torch.int32)
    qkv = torch.zeros(3, H, 400, 64, dtype=torch.float16)
    qkv[..., :dh] = torch.randn(3, H, 400, dh, generator=g).half()
    qkv = qkv.to(DEV)
    kv_off, kv_len = cu[:-1].view(-1, 1).contiguous(), lens.view(-1, 1).contiguous()
    scale = dh**-0.5
    out = k.flash_attn_fwd(qkv[0], qkv[1:2], qkv[2:3], cu.to(DEV), kv_off.to(DEV), kv_len.to(DEV), 300, scale,
                           head_dim=dh)
    assert out.shape == (400, H * dh)
    ref = _attn_ref(qkv[0], qkv[1:2], qkv[2:3], cu, kv_off, kv_len, scale, dh=dh)
    assert float((out[:377].float() - ref[:377]).abs().max()) < 4e-3


@pytest.mark.parametrize("dh,H", [(128, 2), (96, 3), (256, 2), (160, 1)])
@pytest.mark.parametrize("causal", [False, True])
def test_flash_attention_large_heads(cuda_pkg, dh, H, causal):
    """Head dims above 64: rows zero-padded to 128 or 256 halves (one query tile
    per CTA; 64-key tiles at head dim 256), ragged and empty samples."""
    k = cuda_pkg.kernels
    P = k.head_pad(dh)
    g = torch.Generator().manual_seed(dh * 10 + H + int(causal))
    lengths = [300, 1, 0, 129, 700]
    lens = torch.tensor(lengths, dtype=torch.int32)
    cu = torch.zeros(len(lengths) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    n = int(cu[-1])
    rows = n + 64
    qkv = torch.zeros(3, H, rows, P, dtype=torch.float16)
    qkv[..., :dh] = torch.randn(3, H, rows, dh, generator=g).half()
    qkv[:, :, n:] = float("nan")  # slack rows must never leak in
    qkv = qkv.to(DEV)
    kv_off, kv_len = cu[:-1].view(-1, 1).contiguous(), lens.view(-1, 1).contiguous()
    scale = dh**-0.5
    out = k.flash_attn_fwd(qkv[0], qkv[1:2], qkv[2:3], cu.to(DEV), kv_off.to(DEV), kv_len.to(DEV),
                           max(lengths), scale, causal=causal, head_dim=dh)
    assert out.shape == (rows, H * dh)
    ref = _attn_ref(qkv[0], qkv[1:2], qkv[2:3], cu, kv_off, kv_len, scale, causal=causal, dh=dh)
    assert torch.isfinite(out[:n].float()).all()
    assert float((out[:n].float() - ref[:n]).abs().max()) < 4e-3


def test_flash_attention_head_groups_into_strided_context(cuda_pkg):
    """Attention run per head group straight into its columns of the full
    context (row stride = all heads), as the context-parallel path does while
    later groups' K/V are still arriving: equal to one call over all heads."""
    k = cuda_pkg.kernels
    g = torch.Generator().manual_seed(5)
    H, dh = 8, 64
    lens = torch.tensor([300, 0, 77, 129], dtype=torch.int32)
    cu = torch.zeros(5, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    rows = int(cu[-1])
    qkv = torch.randn(3, H, rows, 64, generator=g).half().to(DEV)
    kv_off, kv_len = cu[:-1].view(-1, 1).contiguous().to(DEV), lens.view(-1, 1).contiguous().to(DEV)
    cud = cu.to(DEV)
    full = k.flash_attn_fwd(qkv[0], qkv[1:2], qkv[2:3], cud, kv_off, kv_len, 300, 0.125)
    ctx = torch.full((rows, H * dh), float("nan"), dtype=torch.float16, device=DEV)
    for h0 in range(0, H, 2):
        k.flash_attn_fwd(qkv[0, h0:h0 + 2], qkv[1:2, h0:h0 + 2].contiguous(), qkv[2:3, h0:h0 + 2].contiguous(),
                         cud, kv_off, kv_len, 300, 0.125, out=ctx[:, h0 * dh:(h0 + 2) * dh])
    assert torch.equal(ctx, full)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("dh", [64, 40, 128])
def test_flash_attention_split_and_merge(cuda_pkg, causal, dh):
    """Attention split over two launches as context parallelism runs it: the
    rank's own key segment first (part_mode 1: fp32 partial + log2-sum-exp),
    then the other segments (part_mode 2: merged into ctx).  Non-causal: the
    other segments are segments 0 and 2; causal: the own segment is causal in
    local positions and only the earlier segment 0 follows, unmasked.  Equals
    one softmax over all keys."""
    k = cuda_pkg.kernels
    g = torch.Generator().manual_seed(17 + dh + causal)
    H, P = 3, k.head_pad(dh)
    seg_rows = 700
    lens = [650, 512, 300]   # keys per segment; own segment = 1 (q rows = its tokens)
    nq = lens[1]
    kv = torch.zeros(3, 2, H, seg_rows, P)
    kv[..., :dh] = torch.randn(3, 2, H, seg_rows, dh, generator=g)
    kv = kv.half().to(DEV)
    q = kv[1, 0].clone()     # the own tokens' queries: [H, seg_rows, P]
    q[:, :, :dh] = torch.randn(H, seg_rows, dh, generator=g).half().to(DEV)
    q_cu = torch.tensor([0, nq], dtype=torch.int32, device=DEV)
    scale = dh ** -0.5
    part_o = torch.empty(seg_rows, H * dh, dtype=torch.float32, device=DEV)
    part_lse = torch.empty(seg_rows, H, dtype=torch.float32, device=DEV)
    own_off = torch.zeros(1, 1, dtype=torch.int32, device=DEV)
    own_len = torch.tensor([[lens[1]]], dtype=torch.int32, device=DEV)
    assert k.flash_attn_fwd(q, kv[1:2, 0], kv[1:2, 1], q_cu, own_off, own_len, nq, scale, causal=causal,
                            head_dim=dh, part_o=part_o, part_lse=part_lse, part_mode=1) is None
    remote = [lens[0], 0, 0] if causal else [lens[0], 0, lens[2]]
    out = k.flash_attn_fwd(q, kv[:, 0], kv[:, 1], q_cu, torch.zeros(1, 3, dtype=torch.int32, device=DEV),
                           torch.tensor([remote], dtype=torch.int32, device=DEV), nq, scale, head_dim=dh,
                           part_o=part_o, part_lse=part_lse, part_mode=2)
    # reference: keys = segment 0, segment 1 (own), segment 2 (non-causal only)
    segs = [0, 1] if causal else [0, 1, 2]
    kk = torch.cat([kv[s, 0, :, : lens[s], :dh].float() for s in segs], 1)
    vv = torch.cat([kv[s, 1, :, : lens[s], :dh].float() for s in segs], 1)
    sc = q[:, :nq, :dh].float() @ kk.transpose(1, 2) * scale
    if causal:
        qp = lens[0] + torch.arange(nq, device=DEV)[:, None]
        kp = torch.arange(kk.shape[1], device=DEV)[None, :]
        sc = sc.masked_fill(kp > qp, float("-inf"))
    ref = (torch.softmax(sc, -1) @ vv).transpose(0, 1).reshape(nq, H * dh)
    err = (out[:nq].float() - ref).abs()
    assert torch.isfinite(out[:nq].float()).all()
    assert float(err.max()) < 4e-3, float(err.max())
    # the partial alone is attention over the own keys, its lse the log2 denominator
    so = q[:, :nq, :dh].float() @ kv[1, 0, :, : lens[1], :dh].float().transpose(1, 2) * scale
    if causal:
        so = so.masked_fill(torch.arange(lens[1], device=DEV)[None, :] > torch.arange(nq, device=DEV)[:, None],
                            float("-inf"))
    lse_ref = torch.logsumexp(so, -1) / 0.6931471805599453  # natural log -> log2
    assert float((part_lse[:nq] - lse_ref.transpose(0, 1)).abs().max()) < 2e-3
