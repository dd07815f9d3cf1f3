"""kvbp_decode_gemm vs. a plain PyTorch fp32 reference of the same op.

Reference op: out = bf16(X @ W^T) with X, W bf16 and fp32 accumulation.  With the norm
prologue X = bf16((h * inv_rms) * w_norm), inv_rms = 1/sqrt(mean(h^2) + eps) (fp32).
Residual epilogue: h <- bf16(h + bf16(acc)), plus per-128-column sums of squares of the
new h.  SwiGLU epilogue: act = bf16(bf16(g * bf16(sigmoid(g))) * u), g/u = bf16 outputs.

Tolerance: the kernel accumulates K in a different order (mma tiles, split-K partials),
so an output may land on the neighbouring bf16 value: >= 99 % of outputs bit-identical,
the rest within 2 bf16 ulps (relative 2^-7).  Split-K results are deterministic.
Weights go through kvbp_pack_weight first (the layout the kernel streams).
"""

import math

import pytest
import torch

from kvcacheboundaryprotection_b200 import build, capi
from kvcacheboundaryprotection_b200.engine import interleave_gate_up, pack_weight, unpack_weight

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    build.build()
    capi.lib()


def _close(got, ref):
    got, ref = got.float(), ref.float()
    exact = (got == ref).float().mean().item()
    rel = ((got - ref).abs() / ref.abs().clamp_min(1e-3)).max().item()
    assert exact >= 0.99, exact
    assert rel <= 2.0**-6, rel


def _run(epi, M, N, K, splits, norm=False, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    W = (torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    out_cols = N // 2 if epi == 2 else N
    out = torch.zeros(M, out_cols, dtype=torch.bfloat16, device="cuda")
    if epi == 1:
        out = torch.randn(M, N, generator=g, device="cuda").to(torch.bfloat16)
    h_before = out.clone()
    nw = (1 + 0.1 * torch.randn(K, generator=g, device="cuda")).to(torch.bfloat16) if norm else None
    ss = (x.float() ** 2).sum(1)
    ss_parts = torch.zeros(1, 32, device="cuda")
    ss_parts[0, :M] = ss
    ss_out = torch.full((N // 128, 32), 7.0, device="cuda")  # every entry is written
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    L = capi.lib()
    st = torch.cuda.current_stream().cuda_stream
    Wp = pack_weight(W)
    capi.check(
        L.kvbp_decode_gemm(st, epi, M, N, K, Wp.data_ptr(), x.data_ptr(), K, ss_parts.data_ptr() if norm else None,
                           1, nw.data_ptr() if norm else None, 1e-6, out.data_ptr(), out.shape[1],
                           ss_out.data_ptr() if epi == 1 else None, splits, err.data_ptr()),
        "gemm",
    )
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    xin = x
    if norm:
        inv = 1.0 / torch.sqrt(ss / K + 1e-6)
        xin = ((x.float() * inv[:, None]) * nw.float()).to(torch.bfloat16)
    acc = xin.float() @ W.float().t()
    return W, x, xin, acc, out, h_before, ss_out


def test_pack_unpack_round_trip_and_layout():
    g = torch.Generator(device="cuda").manual_seed(1)
    N, K = 384, 512
    W = torch.randn(N, K, generator=g, device="cuda").to(torch.bfloat16)
    Wp = pack_weight(W)
    assert torch.equal(unpack_weight(Wp), W)
    # element (n, k) -> block (n/128, k/128), half (k%128)/64, row n%128, chunk ((k%64)/8)^(n%8)
    flat = Wp.view(-1).cpu()
    Wc = W.cpu()
    for n, k in [(0, 0), (1, 8), (7, 63), (129, 200), (383, 511), (250, 77)]:
        blk = (n // 128) * (K // 128) + k // 128
        half = (k % 128) // 64
        off = ((blk * 2 + half) * 128 + n % 128) * 64 + ((((k % 64) // 8) ^ (n % 8)) * 8) + k % 8
        assert flat[off] == Wc[n, k], (n, k)


@pytest.mark.parametrize("M", [1, 7, 16, 17, 32])
@pytest.mark.parametrize("splits", [1, 3, 8])
def test_plain(M, splits):
    _, _, _, acc, out, _, _ = _run(0, M, 512, 1024, splits)
    _close(out, acc.to(torch.bfloat16))


@pytest.mark.parametrize("M", [16, 20, 32])  # 17..32 rows run the tcgen05 main loop
@pytest.mark.parametrize("splits", [1, 8])
def test_plain_with_norm_prologue(M, splits):
    _, _, _, acc, out, _, _ = _run(0, M, 4608, 3584, splits, norm=True, seed=3)
    _close(out, acc.to(torch.bfloat16))


@pytest.mark.parametrize("M,splits", [(16, 8), (5, 1), (32, 4), (16, 5), (3, 7), (32, 16)])
def test_residual_epilogue(M, splits):
    _, _, _, acc, out, h0, ss_out = _run(1, M, 3584, 2048, splits, seed=5)
    ref = (h0.float() + acc.to(torch.bfloat16).float()).to(torch.bfloat16)
    # near cancellation a one-ulp difference of bf16(acc) is large relative to h + acc:
    # bound the error by the operands' magnitude instead
    scale = h0.float().abs() + acc.abs()
    assert ((out.float() - ref.float()).abs() <= 2.0**-7 * scale + 1e-6).all()
    assert (out == ref).float().mean().item() >= 0.99
    ss_ref = (out.float() ** 2).view(M, 28, 128).sum(-1).t()  # [tiles][M]
    assert torch.allclose(ss_out[:, :M], ss_ref, rtol=1e-5, atol=1e-5)
    assert (ss_out[:, M:] == 0).all()


@pytest.mark.parametrize("M,splits", [(3, 1), (16, 1), (16, 4), (32, 2)])
def test_swiglu_epilogue_with_norm(M, splits):
    g = torch.Generator(device="cuda").manual_seed(9)
    F, H = 256, 512
    Wg = (torch.randn(F, H, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    Wu = (torch.randn(F, H, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    Wil = interleave_gate_up(Wg, Wu)
    h = torch.randn(M, H, generator=g, device="cuda").to(torch.bfloat16)
    nw = torch.ones(H, dtype=torch.bfloat16, device="cuda")
    ss = torch.zeros(1, 32, device="cuda")
    ss[0, :M] = (h.float() ** 2).sum(1)
    act = torch.zeros(M, F, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    L = capi.lib()
    Wp = pack_weight(Wil)
    capi.check(L.kvbp_decode_gemm(torch.cuda.current_stream().cuda_stream, 2, M, 2 * F, H, Wp.data_ptr(), h.data_ptr(), H,
                                  ss.data_ptr(), 1, nw.data_ptr(), 1e-6, act.data_ptr(), F, None, splits,
                                  err.data_ptr()), "gemm")
    torch.cuda.synchronize()
    inv = 1.0 / torch.sqrt((h.float() ** 2).mean(1) + 1e-6)
    x = ((h.float() * inv[:, None]) * nw.float()).to(torch.bfloat16).float()
    gv = (x @ Wg.float().t()).to(torch.bfloat16).float()
    uv = (x @ Wu.float().t()).to(torch.bfloat16).float()
    sig = torch.sigmoid(gv).to(torch.bfloat16).float()
    ref = ((gv * sig).to(torch.bfloat16).float() * uv).to(torch.bfloat16)
    _close(act, ref)


def test_split_k_is_deterministic():
    outs = [_run(0, 16, 3584, 18944, 8, seed=11)[4] for _ in range(2)]
    assert torch.equal(outs[0], outs[1])


def test_bad_split_count_is_rejected():
    L = capi.lib()
    t = torch.zeros(128 * 256, dtype=torch.bfloat16, device="cuda")
    o = torch.zeros(128, dtype=torch.bfloat16, device="cuda")
    for sp in (0, 3, 17):  # K = 256 allows at most 2 splits
        rc = L.kvbp_decode_gemm(torch.cuda.current_stream().cuda_stream, 0, 1, 128, 256, t.data_ptr(), t.data_ptr(),
                                256, None, 0, None, 1e-6, o.data_ptr(), 128, None, sp, None)
        assert rc != 0


@pytest.mark.parametrize("Hq,Hkv,K,M,splits,bias,qk_norm", [(28, 4, 3584, 16, 7, True, False),
                                                             (16, 8, 1024, 5, 3, False, True),
                                                             (8, 2, 512, 32, 1, True, True)])
def test_fused_qkv_matches_gemm_plus_rope_scatter(Hq, Hkv, K, M, splits, bias, qk_norm):
    """kvbp_decode_qkv_gemm == kvbp_decode_gemm (plain, norm prologue) followed by
    kvbp_qkv_rope_scatter on the same inputs."""
    from kvcacheboundaryprotection_b200.engine import inv_freq_table

    g = torch.Generator(device="cuda").manual_seed(Hq + K)
    D, S = 128, 40
    N = (Hq + 2 * Hkv) * D
    W = (torch.randn(N, K, generator=g, device="cuda") * 0.03).to(torch.bfloat16)
    Wp = pack_weight(W)
    h = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(K, generator=g, device="cuda")).to(torch.bfloat16)
    ss = torch.zeros(1, 32, device="cuda")
    ss[0, :M] = (h.float() ** 2).sum(1)
    b = (0.1 * torch.randn(N, generator=g, device="cuda")).to(torch.bfloat16) if bias else None
    qn = (1 + 0.1 * torch.randn(D, generator=g, device="cuda")).to(torch.bfloat16) if qk_norm else None
    kn = (1 + 0.1 * torch.randn(D, generator=g, device="cuda")).to(torch.bfloat16) if qk_norm else None
    inv = torch.from_numpy(inv_freq_table(D, 1e6)).cuda()
    pos = torch.randint(0, 5000, (M,), generator=g, device="cuda", dtype=torch.int32)
    ws = torch.randperm(S, generator=g, device="cuda")[:M].to(torch.int32) if M <= S else None
    if ws is None:
        ws = (torch.arange(M, device="cuda", dtype=torch.int32) % S)
    ws[0] = -1  # an evicted position: nothing stored
    kc0 = torch.randn(M, Hkv, S, D, generator=g, device="cuda").to(torch.bfloat16)
    vc0 = torch.randn(M, Hkv, S, D, generator=g, device="cuda").to(torch.bfloat16)
    L = capi.lib()
    st = torch.cuda.current_stream().cuda_stream
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    P = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    # reference path: plain GEMM, then the standalone epilogue kernel
    qkv = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    q1 = torch.zeros(M, Hq, D, dtype=torch.bfloat16, device="cuda")
    kc1, vc1 = kc0.clone(), vc0.clone()
    capi.check(L.kvbp_decode_gemm(st, 0, M, N, K, Wp.data_ptr(), h.data_ptr(), K, ss.data_ptr(), 1, nw.data_ptr(),
                                  1e-6, qkv.data_ptr(), N, None, splits, err.data_ptr()), "gemm")
    capi.check(L.kvbp_qkv_rope_scatter(st, M, 1, Hq, Hkv, D, S, qkv.data_ptr(), N, P(b), P(qn), P(kn), 1e-6,
                                       inv.data_ptr(), pos.data_ptr(), ws.data_ptr(), q1.data_ptr(), kc1.data_ptr(),
                                       vc1.data_ptr(), err.data_ptr()), "rope")
    q2 = torch.zeros_like(q1)
    kc2, vc2 = kc0.clone(), vc0.clone()
    capi.check(L.kvbp_decode_qkv_gemm(st, M, Hq, Hkv, K, Wp.data_ptr(), h.data_ptr(), K, ss.data_ptr(), 1,
                                      nw.data_ptr(), 1e-6, P(b), P(qn), P(kn), inv.data_ptr(), pos.data_ptr(),
                                      ws.data_ptr(), S, q2.data_ptr(), kc2.data_ptr(), vc2.data_ptr(), splits,
                                      err.data_ptr()), "qkv_gemm")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    if not qk_norm:
        assert torch.equal(q1, q2) and torch.equal(kc1, kc2) and torch.equal(vc1, vc2)
    else:  # the head norm sums in another order: rare one-ulp differences
        for a_, b_ in ((q1, q2), (kc1, kc2), (vc1, vc2)):
            assert (a_ == b_).float().mean().item() >= 0.99
            assert ((a_.float() - b_.float()).abs() <= 2.0**-7 * a_.float().abs() + 1e-6).all()
    # untouched slots keep their contents; the evicted row stored nothing
    mask = torch.ones(M, S, dtype=torch.bool, device="cuda")
    rows = torch.arange(M, device="cuda")
    mask[rows[ws >= 0], ws[ws >= 0].long()] = False
    assert torch.equal(kc2.permute(0, 2, 1, 3)[mask], kc0.permute(0, 2, 1, 3)[mask])
