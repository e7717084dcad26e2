"""Write path and dequantizer on the GPU: bit-exact against the reference/oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import hq4_oracle as O

pytestmark = pytest.mark.gpu


def _bf16_from_bits(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16).to(device)


def _codes_np(q) -> np.ndarray:
    return q.data.cpu().numpy().view(np.uint8)


def _scales_bits(q) -> np.ndarray:
    return q.scale.cpu().view(torch.int16).numpy().view(np.uint16)


def test_encode_matches_reference_fixture(cuda, golden_encode):
    from asterq.kv import quantize_tensor

    x = _bf16_from_bits(golden_encode["enc_x_bits"], cuda)
    q = quantize_tensor(x, "hadamard_int4", group_size=64)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_codes_np(q), golden_encode["enc_codes"])
    np.testing.assert_array_equal(_scales_bits(q).reshape(x.shape[0], -1), golden_encode["enc_scales"].view(np.uint16))
    assert q.padded_dim == 512 and q.group_size == 64 and q.scheme == "hadamard_int4"
    assert q.scale.shape == (x.shape[0], 8, 1) and q.data.shape == (x.shape[0], 256)


@pytest.mark.parametrize("scheme", ["hadamard_int4", "int4", "int8"])
def test_reference_test_case_48_dims_group16(cuda, golden_encode, scheme):
    """tests/test_quantization.py:8-16 of the reference: [2, 7, 48] bf16, group 16."""
    from asterq.kv import dequantize_tensor, quantize_tensor

    x = _bf16_from_bits(golden_encode["small_x_bits"], cuda)
    q = quantize_tensor(x, scheme, group_size=16)
    np.testing.assert_array_equal(_codes_np(q), golden_encode[f"small_{scheme}_codes"].view(np.uint8))
    np.testing.assert_array_equal(_scales_bits(q), golden_encode[f"small_{scheme}_scales"].view(np.uint16))
    restored = dequantize_tensor(q, dtype=x.dtype)
    assert restored.shape == x.shape
    if scheme != "int8":
        assert float((restored.float() - x.float()).square().mean().sqrt()) < 0.18
    assert q.num_bytes < x.numel() * x.element_size()


def test_round_half_even_ties(cuda, golden_encode):
    from asterq.kv import quantize_tensor

    x = _bf16_from_bits(golden_encode["tie_x_bits"], cuda)
    q = quantize_tensor(x, "int4", group_size=16)
    np.testing.assert_array_equal(_codes_np(q), golden_encode["tie_int4_codes"])


@pytest.mark.parametrize("src_dtype", [torch.bfloat16, torch.float32, torch.float16])
def test_encode_bit_exact_vs_oracle_random(cuda, src_dtype):
    from asterq.kv import quantize_tensor
    from asterq.synth import outlier_channels

    g = torch.Generator(device=cuda).manual_seed(11)
    x = torch.randn(20000, 512, generator=g, device=cuda)
    x[:, outlier_channels(11).to(cuda)] *= 20
    x = x.to(src_dtype)
    q = quantize_tensor(x, "hadamard_int4", group_size=64)
    ref = O.quantize(x.float().cpu().numpy(), "hadamard_int4", 64)
    np.testing.assert_array_equal(_codes_np(q), ref.data)
    np.testing.assert_array_equal(_scales_bits(q), ref.scale.view(np.uint16))


@pytest.mark.parametrize("dim,group", [(512, 32), (512, 16), (256, 64), (128, 64), (96, 64), (64, 16)])
def test_encode_other_geometries(cuda, dim, group):
    """Production configs use latent 96 (padded to 128, kv.py:99-100)."""
    from asterq.kv import quantize_tensor

    g = torch.Generator(device=cuda).manual_seed(dim + group)
    x = torch.randn(3000, dim, generator=g, device=cuda).to(torch.bfloat16)
    q = quantize_tensor(x, "hadamard_int4", group_size=group)
    ref = O.quantize(x.float().cpu().numpy(), "hadamard_int4", group)
    np.testing.assert_array_equal(_codes_np(q), ref.data)
    np.testing.assert_array_equal(_scales_bits(q), ref.scale.view(np.uint16))


def test_encode_strided_rows_and_batch_dims(cuda):
    """Row views of a wider tensor (e.g. a hot page slice) and [B, S, L] inputs."""
    from asterq.kv import quantize_tensor

    g = torch.Generator(device=cuda).manual_seed(5)
    wide = torch.randn(3, 700, 640, generator=g, device=cuda).to(torch.bfloat16)
    x = wide[..., :512]
    q = quantize_tensor(x, "hadamard_int4", group_size=64)
    ref = O.quantize(x.float().cpu().numpy(), "hadamard_int4", 64)
    assert q.data.shape == (3, 700, 256) and q.scale.shape == (3, 700, 8, 1)
    np.testing.assert_array_equal(_codes_np(q), ref.data)


@pytest.mark.parametrize("n", [1, 7, 9, 63, 65, 8 * 8 * 3 + 5])
def test_encode_extreme_magnitudes_and_ragged_tiles(cuda, n):
    """512-value rows in every magnitude regime of the division shortcuts, in
    tiles of 8 tokens with a ragged last tile: zero rows, absmax far below 2^-98
    (codes 0 whatever the quotient), rows whose transform absmax exceeds 2^119
    (the tile switches to IEEE divisions), half-zero rows and constant rows."""
    from asterq.kv import quantize_tensor

    g = torch.Generator(device=cuda).manual_seed(17 + n)
    x = torch.randn(max(n, 12), 512, generator=g, device=cuda)
    x[0] = 0.0
    x[1] *= 1e-30
    x[2] *= 1e-36
    x[3] *= 1e35
    x[4, :64] *= 1e34
    x[5, ::2] = 0.0
    x[6] = 1.0
    x[7] = -3.0
    x[8, 7] = 2.0**60
    x = x[:n].to(torch.bfloat16)
    for group in (64, 32, 16):
        q = quantize_tensor(x, "hadamard_int4", group_size=group)
        ref = O.quantize(x.float().cpu().numpy(), "hadamard_int4", group)
        np.testing.assert_array_equal(_codes_np(q), ref.data)
        np.testing.assert_array_equal(_scales_bits(q), ref.scale.view(np.uint16))


def test_encode_near_ties_take_the_exact_path(cuda):
    """Rows whose normalized transform holds values at (or within rounding of)
    k + 1/2 scale steps: x = a e_0 + b e_1 transforms to (a + b) / c and
    (a - b) / c, and (a - b) / (a + b) = (2k + 1) / 14 puts the smaller one at
    code k + 1/2.  The candidate-and-check rounding must hand these tiles to the
    exact double division."""
    from asterq.kv import quantize_tensor

    g = torch.Generator(device=cuda).manual_seed(29)
    x = torch.randn(37, 512, generator=g, device=cuda)
    for k in range(7):
        a, b = (14 + 2 * k + 1) / 2, (14 - 2 * k - 1) / 2
        for r, sign in ((2 * k, 1.0), (2 * k + 1, -1.0)):
            x[r] = 0.0
            x[r, 0], x[r, 1] = sign * a, b
    x = x.to(torch.bfloat16)
    for group in (64, 32, 16):
        q = quantize_tensor(x, "hadamard_int4", group_size=group)
        ref = O.quantize(x.float().cpu().numpy(), "hadamard_int4", group)
        np.testing.assert_array_equal(_codes_np(q), ref.data)
        np.testing.assert_array_equal(_scales_bits(q), ref.scale.view(np.uint16))


def test_encode_unaligned_rows_take_the_generic_kernel(cuda):
    """A row base that is not 16-byte aligned cannot feed the bulk copies; the
    generic kernel handles it with the same codes."""
    from asterq.kv import quantize_tensor

    g = torch.Generator(device=cuda).manual_seed(23)
    flat = torch.randn(300 * 512 + 1, generator=g, device=cuda).to(torch.bfloat16)
    x = flat[1:].view(300, 512)
    q = quantize_tensor(x, "hadamard_int4", group_size=64)
    ref = O.quantize(x.float().cpu().numpy(), "hadamard_int4", 64)
    np.testing.assert_array_equal(_codes_np(q), ref.data)
    np.testing.assert_array_equal(_scales_bits(q), ref.scale.view(np.uint16))


def test_codec_status_reports_no_timeouts(cuda):
    import ctypes

    from asterq import _lib
    from asterq.kv import quantize_tensor

    quantize_tensor(torch.ones(100, 512, dtype=torch.bfloat16, device=cuda), "hadamard_int4")
    v = ctypes.c_int32(-1)
    assert _lib.load().asterq_codec_status(ctypes.byref(v)) == 0
    assert v.value == 0


def test_encode_c2_full_size_properties(cuda):
    """Config 2 at full size (64 x 4096 tokens): determinism, round-trip error,
    and a bit-exact comparison of a strided sample of rows with the oracle."""
    from asterq.kv import dequantize_tensor, quantize_tensor
    from asterq.synth import outlier_channels

    g = torch.Generator(device=cuda).manual_seed(2)
    x = torch.randn(64, 4096, 512, generator=g, device=cuda)
    x[..., outlier_channels(2).to(cuda)] *= 20
    x = x.to(torch.bfloat16)
    q1 = quantize_tensor(x, "hadamard_int4", group_size=64)
    q2 = quantize_tensor(x, "hadamard_int4", group_size=64)
    assert torch.equal(q1.data, q2.data) and torch.equal(q1.scale, q2.scale)
    sample = x.reshape(-1, 512)[::97]
    ref = O.quantize(sample.float().cpu().numpy(), "hadamard_int4", 64)
    np.testing.assert_array_equal(q1.data.reshape(-1, 256)[::97].cpu().numpy(), ref.data)
    restored = dequantize_tensor(q1, dtype=torch.float32)
    err = (restored - x.float()).square().mean().sqrt() / x.float().square().mean().sqrt()
    assert float(err) < 0.2


@pytest.mark.parametrize("src", ["bf16", "f32"])
def test_float8_write_path_matches_reference_fixture(cuda, golden_encode, src):
    """asterq_quantize with ASTERQ_SCHEME_FLOAT8 writes the bytes of the reference's
    x.to(torch.float8_e4m3fn) (kv.py:85-89) for bf16 and float32 rows, edge values included
    (subnormal ties, 448 < |x| <= 464, beyond 464, infinities, NaN, signed zeros), and
    asterq_dequantize widens them back exactly."""
    from asterq import _lib

    lib = _lib.load()
    if src == "bf16":
        x = _bf16_from_bits(golden_encode["f8_x_bits"], cuda)
        want = golden_encode["f8_codes_bf16"]
    else:
        x = torch.from_numpy(golden_encode["f8_x_f32"]).to(cuda)
        want = golden_encode["f8_codes_f32"]
    n, dim = x.shape
    codes = torch.empty(n, dim, dtype=torch.uint8, device=cuda)
    _lib.check(lib.asterq_quantize(x.data_ptr(), _lib.dtype_code(x.dtype), n, dim, dim, _lib.SCHEME_FLOAT8, 64,
                                   codes.data_ptr(), None, _lib.stream_handle(x.device)))
    np.testing.assert_array_equal(codes.cpu().numpy(), want)
    back = torch.empty(n, dim, dtype=torch.float32, device=cuda)
    _lib.check(lib.asterq_dequantize(codes.data_ptr(), None, n, dim, _lib.SCHEME_FLOAT8, 64, back.data_ptr(),
                                     _lib.DTYPE_F32, dim, _lib.stream_handle(x.device)))
    np.testing.assert_array_equal(back.cpu().numpy(), O.float8_values(want))


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_dequantize_bit_exact(cuda, golden_encode, out_dtype):
    from asterq.kv import QuantizedTensor, dequantize_tensor

    codes = golden_encode["enc_codes"]
    scales = golden_encode["enc_scales"].view(np.float16)
    n = codes.shape[0]
    q = QuantizedTensor(torch.from_numpy(codes).to(cuda), torch.from_numpy(scales.copy()).reshape(n, 8, 1).to(cuda),
                        (n, 512), 512, 64, "hadamard_int4", torch.bfloat16)
    out = dequantize_tensor(q, dtype=out_dtype).cpu()
    ref = O.dequantize(O.Quantized(codes, scales.reshape(n, 8, 1), (n, 512), 512, 64, "hadamard_int4"))
    ref_t = torch.from_numpy(ref).to(out_dtype)
    # rows whose fp16 scale overflowed to inf hold NaN: compare NaN positions, not payload bits
    nan = torch.isnan(ref_t)
    assert torch.equal(torch.isnan(out), nan)
    ibits = torch.int16 if out_dtype != torch.float32 else torch.int32
    assert torch.equal(out.view(ibits)[~nan], ref_t.view(ibits)[~nan])


@pytest.mark.parametrize("n", [2, 16, 64, 128, 512])
def test_fwht_bit_exact(cuda, n):
    from asterq.kv import normalized_fwht

    g = torch.Generator(device=cuda).manual_seed(n)
    x = torch.randn(777, n, generator=g, device=cuda) * 3
    x[0] = 0.0
    x[1] = 1e-38  # subnormal neighbourhood: exercises the IEEE-division fallback
    y = normalized_fwht(x).cpu()
    ref = torch.from_numpy(O.normalized_fwht(x.cpu().numpy()))
    assert torch.equal(y.view(torch.int32), ref.view(torch.int32))


def test_encode_rejects_cpu_tensors():
    from asterq.kv import quantize_tensor

    with pytest.raises(RuntimeError, match="CUDA"):
        quantize_tensor(torch.zeros(4, 512), "hadamard_int4")


def test_encode_empty_input(cuda):
    from asterq.kv import quantize_tensor

    q = quantize_tensor(torch.zeros(0, 512, dtype=torch.bfloat16, device=cuda), "hadamard_int4")
    assert q.data.shape == (0, 256) and q.scale.shape == (0, 8, 1)
