"""tcgen05 prefill projection (kvbp_prefill_gemm) vs. a plain PyTorch fp32 reference of the
same op: out = bf16(X . W^T) with fp32 accumulation, W read from the packed layout.

Tolerance: the fp32 sum runs in another order (tensor-core K steps of 16 vs. the
reference GEMM), so an output may land on the neighbouring bf16 value: >= 99 % of the
elements bit-identical, the rest within 2 bf16 ulps (1e-4 absolute near zero).  The SwiGLU epilogue applies the
reference's rounding points to the bf16 gate / up outputs (as the decode GEMM does)."""

import pytest
import torch

from kvcacheboundaryprotection_b200 import build, capi
from kvcacheboundaryprotection_b200.engine import interleave_gate_up, pack_weight

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib():
    build.build()


def _check(got, want):
    """>= 99 % bit-identical; the rest within 2 bf16 ulps, or within 1e-4 absolute where the
    sum cancels to a value far below its terms (outputs are O(1) here; the fp32 sum of
    hundreds of O(0.02) terms carries ~1e-6 of absolute rounding, a large relative error
    on a result near zero)."""
    got, want = got.float(), want.float()
    d = (got - want).abs()
    ulp = torch.finfo(torch.bfloat16).eps * want.abs()
    assert (d == 0).float().mean().item() >= 0.99, (d == 0).float().mean().item()
    assert (d <= 2 * ulp + 1e-4).all(), d.max().item()


def _run(epi, x, wp, N, out_cols):
    M, K = x.shape
    out = torch.full((M, out_cols), float("nan"), dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    capi.check(capi.lib().kvbp_prefill_gemm(torch.cuda.current_stream().cuda_stream, epi, M, N, K, wp.data_ptr(),
                                            x.data_ptr(), x.stride(0), out.data_ptr(), out.stride(0), err.data_ptr()),
               "prefill_gemm")
    torch.cuda.synchronize()
    assert int(err.item()) == 0, capi.decode_dev_errors(int(err.item()))
    return out


@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (300, 1152, 896), (1024, 4608, 3584), (4096, 3584, 18944 // 4),
                                   (513, 2560, 2048)])
def test_prefill_gemm_plain(M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M + N)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    out = _run(0, x, pack_weight(w), N, N)
    _check(out, (x.float() @ w.float().t()).to(torch.bfloat16))


@pytest.mark.parametrize("M,F,K", [(200, 1024, 512), (1024, 2816, 1024), (777, 18944 // 4, 3584)])
def test_prefill_gemm_swiglu(M, F, K):
    """The SwiGLU epilogue applies act = bf16(bf16(g * bf16(sigmoid(g))) * u) to the kernel's own
    bf16 gate / up outputs: against the plain epilogue's outputs of the same packed weights
    (same accumulation order) finished in torch it is bit-identical up to the sigmoid's
    rounding (torch's exp vs. CUDA's expf: one bf16 ulp, rarely).  The plain outputs
    themselves are held to the fp32 reference above."""
    from kvcacheboundaryprotection_b200.engine import deinterleave_gate_up

    g = torch.Generator(device="cuda").manual_seed(M + F)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    wg = (torch.randn(F, K, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    wu = (torch.randn(F, K, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    wp = pack_weight(interleave_gate_up(wg, wu))
    out = _run(2, x, wp, 2 * F, F)
    gu = deinterleave_gate_up(_run(0, x, wp, 2 * F, 2 * F)).float()
    gate, up = gu[:, :F], gu[:, F:]
    _check(torch.cat([gate, up], 1).to(torch.bfloat16),
           torch.cat([x.float() @ wg.float().t(), x.float() @ wu.float().t()], 1).to(torch.bfloat16))
    sig = (1.0 / (1.0 + torch.exp(-gate))).to(torch.bfloat16).float()
    want = ((gate * sig).to(torch.bfloat16).float() * up).to(torch.bfloat16).float()
    d = (out.float() - want).abs()
    assert (d == 0).float().mean().item() >= 0.999
    assert (d <= torch.finfo(torch.bfloat16).eps * want.abs() * 2 + 1e-6).all(), d.max().item()


def test_prefill_gemm_rejects_bad_shapes():
    L = capi.lib()
    st = torch.cuda.current_stream().cuda_stream
    x = torch.zeros(4, 128, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(128, 128, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(4, 128, dtype=torch.bfloat16, device="cuda")
    assert L.kvbp_prefill_gemm(st, 0, 4, 100, 128, w.data_ptr(), x.data_ptr(), 128, out.data_ptr(), 128, None) != 0
    assert L.kvbp_prefill_gemm(st, 1, 4, 128, 128, w.data_ptr(), x.data_ptr(), 128, out.data_ptr(), 128, None) != 0


@pytest.mark.parametrize("M,N,K", [(300, 1152, 896), (1024, 3584, 4736), (513, 2048, 1024)])
def test_prefill_gemm_fp32_partials(M, N, K):
    """Epilogue 3 writes the fp32 accumulators (the row-parallel partial sums of tensor
    parallelism): within fp32 rounding of the fp32 reference product (the K-step order
    differs), and rounding them to bf16 gives the plain epilogue's output."""
    g = torch.Generator(device="cuda").manual_seed(M + K)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    wp = pack_weight(w)
    out = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    capi.check(capi.lib().kvbp_prefill_gemm(torch.cuda.current_stream().cuda_stream, 3, M, N, K, wp.data_ptr(),
                                            x.data_ptr(), x.stride(0), out.data_ptr(), out.stride(0), err.data_ptr()),
               "prefill_gemm")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = x.float() @ w.float().t()
    scale = (x.float().abs() @ w.float().abs().t())  # bound of the terms' magnitudes
    assert ((out - ref).abs() <= 1e-4 * scale + 1e-6).all()
    plain = _run(0, x, wp, N, N)
    assert torch.equal(out.to(torch.bfloat16), plain)
