"""Pin the numpy oracle against golden vectors produced by the reference.

The fixtures come from tests/golden/make_golden.py (the reference's own
liteweight.quantize and an HF LlamaForCausalLM decode). Integer codes, packed
bytes and dequantized fp16 weights must be bit-exact; fp32-accumulated matmul
outputs may differ by the accumulation order, so they are compared at one
fp16 ulp; decode logits use the row-scaled tolerance of the kernels.
"""

import numpy as np
import pytest

from oracle import llama as ol
from oracle import quant as oq


@pytest.fixture(scope="module")
def qg(golden_dir):
    return dict(np.load(golden_dir / "quant_golden.npz"))


def _cases(qg):
    return sorted({k.split("/")[0] for k in qg if "/W" in k or k.endswith("/W")})


def test_fixture_has_cases(qg):
    names = _cases(qg)
    assert "tq_64x256" in names and "ties_i8" in names and "bench_perchan" in names
    assert len(names) >= 10


def test_quantize_bit_exact(qg):
    for name in _cases(qg):
        W, G = qg[f"{name}/W"], int(qg[f"{name}/G"])
        q8, s8 = oq.quantize_int8(W, G)
        q4, s4 = oq.quantize_int4(W, G)
        np.testing.assert_array_equal(q8, qg[f"{name}/q8"], err_msg=name)
        np.testing.assert_array_equal(s8.view(np.uint16), qg[f"{name}/s8"].view(np.uint16), err_msg=name)
        np.testing.assert_array_equal(q4, qg[f"{name}/q4"], err_msg=name)
        np.testing.assert_array_equal(s4.view(np.uint16), qg[f"{name}/s4"].view(np.uint16), err_msg=name)


def test_dequantize_bit_exact(qg):
    for name in _cases(qg):
        if f"{name}/dq8" not in qg:
            continue
        G = int(qg[f"{name}/G"])
        d8 = oq.dequantize_int8(qg[f"{name}/q8"], qg[f"{name}/s8"], G)
        d4 = oq.dequantize_int4(qg[f"{name}/q4"], qg[f"{name}/s4"], G)
        np.testing.assert_array_equal(d8.view(np.uint16), qg[f"{name}/dq8"].view(np.uint16), err_msg=name)
        np.testing.assert_array_equal(d4.view(np.uint16), qg[f"{name}/dq4"].view(np.uint16), err_msg=name)


def test_all_codes_bit_exact(qg):
    d4 = oq.dequantize_int4(qg["codes4/q"], qg["codes4/s"], 128)
    np.testing.assert_array_equal(d4.view(np.uint16), qg["codes4/dq"].view(np.uint16))
    d8 = oq.dequantize_int8(qg["codes8/q"], qg["codes8/s"], 128)
    np.testing.assert_array_equal(d8.view(np.uint16), qg["codes8/dq"].view(np.uint16))
    # every nibble value appears, including -8
    codes = oq.unpack_int4(qg["codes4/q"])
    assert set(np.unique(codes)) == set(range(-8, 8))
    assert qg["codes8/q"].min() == -128


def test_round_half_even_ties(qg):
    q8 = qg["ties_i8/q8"][0]
    # w/scale = +-(i + 0.5): half-to-even rounding gives the even neighbour
    got = oq.quantize_int8(qg["ties_i8/W"], 128)[0][0]
    np.testing.assert_array_equal(got, q8)
    assert np.all(np.abs(q8[1:]) % 2 == 0)


def test_fakequant_matmul_close(qg):
    """Both sides sum K fp32 products in different orders: allow one fp16 ulp
    plus a probabilistic fp32 accumulation bound 4*sqrt(K)*2^-24*sum|a||w|."""
    for name in _cases(qg):
        if f"{name}/act" not in qg:
            continue
        act, W, G = qg[f"{name}/act"], qg[f"{name}/W"], int(qg[f"{name}/G"])
        for out, fn, deq in (("out8", oq.fakequant_matmul, lambda: oq.dequantize_int8(*oq.quantize_int8(W, G), G)),
                             ("out4", oq.fakequant_matmul_int4, lambda: oq.dequantize_int4(*oq.quantize_int4(W, G), G))):
            got = fn(act, W, G).astype(np.float32)
            ref = qg[f"{name}/{out}"].astype(np.float32)
            big = np.maximum(np.abs(ref), np.abs(got)).astype(np.float16)
            ulp = np.abs(np.spacing(big)).astype(np.float32)
            mag = np.abs(act.astype(np.float64)) @ np.abs(deq().astype(np.float64)).T
            tol = ulp + 4 * np.sqrt(act.shape[1]) * 2.0 ** -24 * mag
            assert np.all(np.abs(got - ref) <= tol), (name, out, np.abs(got - ref).max())


def test_packed_matmul_equals_fakequant(qg):
    name = "tk_M3_K256_N40_G128"
    act, G = qg[f"{name}/act"], 128
    a = oq.packed_matmul(act, qg[f"{name}/q8"], qg[f"{name}/s8"], G, 8)
    b = oq.fakequant_matmul(act, qg[f"{name}/W"], G)
    np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("fixture", ["llama_tiny_int8.npz", "llama_tiny_int4.npz"])
def test_llama_oracle_matches_hf(golden_dir, fixture):
    d = dict(np.load(golden_dir / fixture))
    w = ol.from_fixture(d)
    ref = d["logits"].astype(np.float32)                 # [T, B, V]
    got = ol.teacher_forced_logits(w, d["prompt"], d["tokens"]).astype(np.float32)
    assert got.shape == ref.shape
    tol = oq.row_tolerance(ref.reshape(-1, ref.shape[-1])).reshape(ref.shape[0], ref.shape[1], 1)
    err = np.abs(got - ref)
    assert np.all(err <= tol), float((err / tol).max())
    # greedy picks along the teacher-forced path
    match = (ol.greedy(got.reshape(-1, got.shape[-1])) == d["tokens"].T.reshape(-1)).mean()
    assert match >= 0.9, match


def test_torch_cpu_restatement_bit_exact(qg):
    """The torch CPU restatement timed as the CPU baseline dequantizes exactly
    like the reference (golden dq arrays) and its matmul equals the oracle's
    fakequant result within the fp32-order bound."""
    import torch
    from oracle import torch_cpu as tc
    for name in _cases(qg):
        if f"{name}/dq8" not in qg:
            continue
        G = int(qg[f"{name}/G"])
        for bits, key in ((8, "8"), (4, "4")):
            q = torch.from_numpy(qg[f"{name}/q{key}"])
            s = torch.from_numpy(qg[f"{name}/s{key}"])
            d = (tc.dequantize_int8 if bits == 8 else tc.dequantize_int4)(q, s, G)
            np.testing.assert_array_equal(d.numpy().view(np.uint16), qg[f"{name}/dq{key}"].view(np.uint16),
                                          err_msg=f"{name} int{bits}")
    d4 = tc.dequantize_int4(torch.from_numpy(qg["codes4/q"]), torch.from_numpy(qg["codes4/s"]), 128)
    np.testing.assert_array_equal(d4.numpy().view(np.uint16), qg["codes4/dq"].view(np.uint16))
    name = "tk_M3_K256_N40_G128"
    act = qg[f"{name}/act"]
    got = tc.quant_linear(torch.from_numpy(act), torch.from_numpy(qg[f"{name}/q4"]),
                          torch.from_numpy(qg[f"{name}/s4"]), 128, 4).numpy().astype(np.float32)
    ref = oq.packed_matmul(act, qg[f"{name}/q4"], qg[f"{name}/s4"], 128, 4).astype(np.float32)
    big = np.maximum(np.abs(ref), np.abs(got)).astype(np.float16)
    assert np.all(np.abs(got - ref) <= np.abs(np.spacing(big)).astype(np.float32) + 1e-6)
