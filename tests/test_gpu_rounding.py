"""bf16 rounding fences on the GPU against the oracle (row a14):
sc_bf16_round restates burn_flex_gmm's bf16_round_to_f32_kernel
(src/wgpu.rs:57-67): round the f32 bit pattern to nearest-even at bit 16 with
no NaN special case, kept in f32.  It must agree bit for bit with
oracle.bf16_round on every input, including ties, NaN payloads, infinities,
subnormals and values that round past the bf16 maximum.  sc_cast (f32 -> bf16
storage) rounds the same way for every non-NaN input and keeps NaN a NaN;
bf16 -> f32 widens exactly."""
import numpy as np
import pytest
import torch

import oracle
from bevy_synth_b200 import flex_gmm as F

from gpu_util import assert_no_fault, to_dev

pytestmark = pytest.mark.gpu


def special_bits() -> np.ndarray:
    one = 0x3F800000
    pats = [
        0x00000000, 0x80000000,                      # +-0
        0x00000001, 0x00007FFF, 0x00008000, 0x00008001, 0x00018000, 0x0000FFFF,  # subnormal ties / rounding
        0x007FFFFF, 0x00800000, 0x00808000, 0x00818000,                           # largest subnormal, smallest normal
        one, one | 0x8000, one | 0x8001, one | 0x7FFF, one | 0x18000, one | 0x28000,  # ties to even around 1.0
        0x7F7F0000, 0x7F7F7FFF, 0x7F7F8000, 0x7F7FFFFF,   # near the bf16 / f32 maximum (ties round up to inf)
        0x7F800000, 0xFF800000,                          # +-inf
        0x7FC00000, 0xFFC00000, 0x7F800001, 0x7F807FFF, 0x7F808000, 0x7FFFFFFF, 0xFF800001,  # NaN payloads
        0xBF808000, 0xBF818000, 0xC2C9A3D7,
    ]
    rng = np.random.default_rng(3)
    rnd = rng.integers(0, 2 ** 32, size=200_000, dtype=np.uint64).astype(np.uint32)
    ties = (rng.integers(0, 2 ** 16, size=20_000, dtype=np.uint64).astype(np.uint32) << 16) | 0x8000
    return np.concatenate([np.array(pats, np.uint32), rnd, ties])


def test_bf16_round_matches_oracle_bits(cuda_device):
    bits = special_bits()
    x = bits.view(np.float32)
    got = F.bf16_round_to_f32(to_dev(x)).cpu().numpy().view(np.uint32)
    exp = oracle.bf16_round(x).view(np.uint32)
    bad = np.nonzero(got != exp)[0]
    assert bad.size == 0, [(hex(bits[i]), hex(got[i]), hex(exp[i])) for i in bad[:8]]
    # the formula's documented corner cases
    assert exp[list(bits).index(0x7F7FFFFF)] == 0x7F800000      # FLT_MAX rounds to +inf
    assert exp[list(bits).index(0x7F800001)] == 0x7F800000      # no NaN special case
    assert exp[list(bits).index(0x3F808000)] == 0x3F800000      # tie to even (down)
    assert exp[list(bits).index(0x3F818000)] == 0x3F820000      # tie to even (up)
    assert_no_fault()


def test_cast_f32_to_bf16_and_back(cuda_device):
    bits = special_bits()
    x = bits.view(np.float32)
    xb = F.cast(to_dev(x), torch.bfloat16)
    back = F.cast(xb, torch.float32).cpu().numpy()
    exp = oracle.bf16_round(x)
    nan_in = np.isnan(x)
    np.testing.assert_array_equal(back.view(np.uint32)[~nan_in], exp.view(np.uint32)[~nan_in])
    assert np.isnan(back[nan_in]).all()
    # bf16 -> f32 is exact: every bf16 bit pattern widens to its upper-half f32
    all_bf16 = np.arange(2 ** 16, dtype=np.uint32).astype(np.uint16)
    t = torch.from_numpy(all_bf16.view(np.int16)).view(torch.bfloat16).to("cuda")
    wide = F.cast(t, torch.float32).cpu().numpy().view(np.uint32)
    finite = ((all_bf16.astype(np.uint32) & 0x7F80) != 0x7F80) | ((all_bf16.astype(np.uint32) & 0x7F) == 0)
    np.testing.assert_array_equal(wide[finite], all_bf16.astype(np.uint32)[finite] << 16)
    assert np.isnan(wide[~finite].view(np.float32)).all()
    assert_no_fault()
