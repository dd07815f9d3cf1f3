"""The prefill attention kernel rounds fp32 values to bf16 precision on the FP32 pipe
(`rnd_bf16` in kvcacheboundaryprotection_b200/csrc/prefill_attn.cu): a Veltkamp split with
sigma = 2^16 + 1,

    g  = RN(65537 * x)
    hi = RN(g + RN(x - g)),

keeps the leading 8 significand bits of x.  These tests check, in IEEE float32 arithmetic
(numpy rounds each operation to nearest-even, as the kernel's `__fmul_rn` / `__fsub_rn` /
`__fadd_rn` do), that hi is exactly the round-to-nearest-even bf16 value of x, ties
included, over whole binades of both signs and against torch's bf16 cast."""

import numpy as np
import pytest
import torch


def veltkamp_bf16(x: np.ndarray) -> np.ndarray:
    s = np.float32(65537.0)
    g = (s * x).astype(np.float32)
    d = (x - g).astype(np.float32)
    return (g + d).astype(np.float32)


def rne_bf16(x: np.ndarray) -> np.ndarray:
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


@pytest.mark.parametrize("biased_exp", [1, 100, 127, 140, 237])
def test_veltkamp_equals_round_to_nearest_even_on_whole_binades(biased_exp):
    mant = np.arange(1 << 23, dtype=np.uint32)
    for sign in (0, 1):
        bits = (np.uint32(sign) << np.uint32(31)) | (np.uint32(biased_exp) << np.uint32(23)) | mant
        x = bits.view(np.float32)
        with np.errstate(over="ignore", invalid="ignore"):
            got = veltkamp_bf16(x)
        want = rne_bf16(x)
        bad = np.flatnonzero(got.view(np.uint32) != want.view(np.uint32))
        assert bad.size == 0, f"exp {biased_exp} sign {sign}: {bad.size} mismatches, first x={x[bad[0]]!r}"


def test_ties_round_to_even():
    # x = 1 + (2k + 1) * 2^-8 lies halfway between two bf16 neighbours
    k = np.arange(128, dtype=np.float32)
    x = (np.float32(1.0) + (2 * k + 1) * np.float32(2.0 ** -8)).astype(np.float32)
    got = veltkamp_bf16(x).view(np.uint32) >> 16
    assert np.all((got & 1) == 0)
    assert np.array_equal(veltkamp_bf16(x), rne_bf16(x))


def test_veltkamp_matches_torch_bf16_cast():
    x = (np.random.default_rng(7).standard_normal(1 << 20) * 37).astype(np.float32)
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(veltkamp_bf16(x).view(np.uint32), want.view(np.uint32))
