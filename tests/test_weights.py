"""Weight ingestion (burn_trellis sparse_decoder_loading.rs): safetensors
container, dtypes, and the reference's validation rules (CPU only)."""
import numpy as np
import pytest

from bevy_synth_b200 import weights as Wt


def _bf16(a):
    u = np.asarray(a, np.float32).view(np.uint32)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


def test_roundtrip_dtypes(tmp_path):
    rng = np.random.default_rng(0)
    a = rng.standard_normal((3, 4)).astype(np.float32)
    b = rng.standard_normal(7).astype(np.float16)
    c = rng.standard_normal((2, 3, 5)).astype(np.float32)
    p = tmp_path / "w.safetensors"
    Wt.write_safetensors(p, {"a": a, "b": b, "c": c}, bf16=("c",))
    st = Wt.read_safetensors(str(p))
    assert st["a"].dtype == "F32" and st["a"].shape == (3, 4)
    np.testing.assert_array_equal(st["a"].data.reshape(3, 4), a)
    assert st["b"].dtype == "F16"
    np.testing.assert_array_equal(st["b"].data, b)
    assert st["c"].dtype == "BF16" and st["c"].shape == (2, 3, 5)
    got = (st["c"].data.astype(np.uint32) << 16).view(np.float32).reshape(2, 3, 5)
    np.testing.assert_array_equal(got, _bf16(c))


def test_validation_messages(tmp_path):
    p = tmp_path / "bad.safetensors"
    Wt.write_safetensors(p, {"conv.weight": np.zeros((8, 3, 3, 3), np.float32), "conv.bias": np.zeros(8, np.float32),
                             "lin.weight": np.zeros((8, 16), np.float32), "lin.bias": np.zeros(4, np.float32),
                             "vec": np.zeros(5, np.float32)})
    st = Wt.read_safetensors(str(p))
    with pytest.raises(Wt.WeightError, match="missing tensor 'nope'"):
        Wt.load_vector(st, "nope", 0, "cpu")
    with pytest.raises(Wt.WeightError, match="expected rank=5, got rank=4"):
        Wt.load_sparse_conv(st, "conv.weight", "conv.bias", 0, 0, "cpu")
    with pytest.raises(Wt.WeightError, match=r"tensor 'lin.bias' expected shape=\[8\], got \[4\]"):
        Wt.load_linear(st, "lin.weight", "lin.bias", 16, 8, "cpu", dtype=None)
    with pytest.raises(Wt.WeightError, match="expected in_channels=32, got 16"):
        Wt.load_linear(st, "lin.weight", "lin.bias", 32, 8, "cpu")
    with pytest.raises(Wt.WeightError, match="expected len=4, got len=5"):
        Wt.load_vector(st, "vec", 4, "cpu")
    v = Wt.load_vector(st, "vec", 5, "cpu")
    assert v.shape == (5,) and float(v.sum()) == 0.0


def test_grouped_conv_rules(tmp_path):
    p = tmp_path / "g.safetensors"
    Wt.write_safetensors(p, {"w": np.zeros((6, 3, 3, 3, 4), np.float32), "b": np.zeros(6, np.float32)})
    st = Wt.read_safetensors(str(p))
    with pytest.raises(Wt.WeightError, match="expected_in=6 is incompatible with in_per_group=4"):
        Wt.load_sparse_conv(st, "w", "b", 6, 6, "cpu")
    with pytest.raises(Wt.WeightError, match=r"incompatible grouped channels \(groups=4, out_channels=6\)"):
        Wt.load_sparse_conv(st, "w", "b", 16, 6, "cpu")
