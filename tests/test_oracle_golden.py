"""Pin the CPU oracle against golden vectors produced by the reference's own kernels.

The fixtures were written by ``tests/golden/make_golden.py``, which runs the
reference ``fp_attention`` / ``fp_chain_<N>`` Triton kernels through the
reference ``execute_plan`` under ``TRITON_INTERPRET=1``.
"""

import numpy as np
import pytest

import oracle
from tests import _golden

ATTN = _golden.names("attn")
CHAIN = _golden.names("chain")


@pytest.mark.parametrize("name", ATTN)
def test_attention_oracle_matches_reference(name):
    meta, a = _golden.load(name)
    out = oracle.attention_fwd(a["q"], a["k"], a["v"], meta["scale"], out_dtype=a["out"].dtype)
    assert out.dtype == a["out"].dtype and out.shape == a["out"].shape
    if meta["dtype"] == "f32":
        np.testing.assert_allclose(out, a["out"], rtol=1e-6, atol=1e-6)
    else:  # one f16 rounding of nearly identical f32 values: at most 1 ulp apart
        np.testing.assert_allclose(out.astype(np.float32), a["out"].astype(np.float32),
                                   rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("name", CHAIN)
def test_chain_oracle_matches_reference(name):
    meta, a = _golden.load(name)
    n = meta["n_args"]
    ops, res = oracle.body_to_program(n, meta["body"])
    ins = [a[f"x{i}"] for i in range(n)]
    fn = oracle.chain_rows if meta["launch"] == "rows" else oracle.chain_flat
    out = fn(ins, ops, res, meta["shape"], a["out"].dtype)
    ref = a["out"]
    has_exp = any(o[0] in ("exp", "softmax") for o in ops)
    if not has_exp:
        # add/mul/scale/relu in f32 with one final rounding: bit-exact
        np.testing.assert_array_equal(out, ref)
    elif meta["dtype"] == "f32":
        np.testing.assert_allclose(out, ref, rtol=1e-6, atol=1e-7)
    else:
        np.testing.assert_allclose(out.astype(np.float32), ref.astype(np.float32), rtol=1e-3, atol=1e-6)


def test_broadcast_operands_equal_expanded_reference():
    """The product passes b, s of the cfg2 chain un-expanded; the oracle broadcast
    must equal the reference run on the expanded operands, bit for bit."""
    meta, a = _golden.load("chain_flat_f16_cfg2_64x256")
    ops, res = oracle.body_to_program(3, meta["body"])
    out = oracle.chain_flat([a["x0"], a["x1_small"], a["x2_small"]], ops, res, meta["shape"], np.float16)
    np.testing.assert_array_equal(out, a["out"])


def test_planted_mistake_is_caught():
    """A scale changed by 1.5x in the oracle must fail against the reference fixture
    (mirrors the reference gate test tests/test_verify_bench.py:241-252)."""
    meta, a = _golden.load("attn_f32_1x2x20x16")
    bad = oracle.attention_fwd(a["q"], a["k"], a["v"], meta["scale"] * 1.5)
    assert not np.allclose(bad, a["out"], rtol=1e-3, atol=1e-3)
