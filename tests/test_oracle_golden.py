"""Pin the oracle: the numpy restatement must reproduce the committed golden
vectors bit-for-bit (gguf-py 0.19.0 and the reference C engine compiled from
source), so that every GPU parity test inherits a pinned checker."""
import os

import numpy as np
import pytest

from oracle import formats as F
from oracle import ops as O

G = os.path.join(os.path.dirname(__file__), "golden")
FM = np.load(os.path.join(G, "formats.npz"))
RO = np.load(os.path.join(G, "ref_ops.npz"))

DEQ_TYPES = [F.Q4_0, F.Q4_1, F.Q5_0, F.Q8_0, F.Q4_K, F.Q5_K, F.Q6_K, F.MXFP4, F.BF16]


@pytest.mark.parametrize("qt", DEQ_TYPES, ids=lambda q: F.NAMES[q])
def test_dequant_matches_gguf_bits(qt):
    raw, exp = FM[f"deq_raw_{qt}"], FM[f"deq_out_{qt}"]
    got = F.dequantize(qt, raw, exp.size)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


@pytest.mark.parametrize("qt", [F.Q4_K, F.Q5_K, F.Q6_K, F.Q8_0], ids=lambda q: F.NAMES[q])
def test_dequant_matches_reference_c_bits(qt):
    got = F.dequantize(qt, FM[f"deq_raw_{qt}"], 512)
    assert np.array_equal(got.view(np.uint32), FM[f"ref_deq_{qt}"].view(np.uint32))


@pytest.mark.parametrize("qt", [F.Q8_0, F.Q4_0, F.MXFP4], ids=lambda q: F.NAMES[q])
def test_quantize_matches_gguf_bytes(qt):
    assert np.array_equal(F.quantize(qt, FM["quant_x"]), FM[f"quant_gguf_{qt}"])


def test_q8_0_activation_quantizer_matches_reference_bytes():
    assert np.array_equal(F.quantize_q8_0(FM["quant_x"]), FM["ref_q8_0_bytes"])


# where the reference's dispatcher is W.x, the fp64 oracle agrees with its fp32 output
@pytest.mark.parametrize("qt", [F.Q8_0, F.Q4_0, F.Q4_1, F.Q5_K, F.MXFP4_REF], ids=lambda q: F.NAMES[q])
def test_gemv_oracle_matches_reference_dispatch(qt):
    n, k, _ = RO["shape"]
    got = O.gemv(RO[f"gemv_w_{qt}"], qt, RO[f"gemv_x_{qt}"], n, k)[0]
    assert O.rel_l2(RO[f"gemv_ref_dispatch_{qt}"], got) < 1e-5


@pytest.mark.parametrize("qt", [F.Q8_0, F.Q4_0, F.Q4_K, F.MXFP4_REF], ids=lambda q: F.NAMES[q])
def test_batch_gemv_oracle_matches_reference(qt):
    n, k, b = RO["shape"]
    got = O.gemv(RO[f"gemv_w_{qt}"], qt, RO[f"bgemv_x_{qt}"], n, k)
    assert O.rel_l2(RO[f"bgemv_ref_{qt}"], got) < 1e-5


@pytest.mark.parametrize("qt", [F.Q4_K, F.Q6_K], ids=lambda q: F.NAMES[q])
def test_reference_dispatch_deviation_is_recorded(qt):
    """The reference's type-12 / type-14 dispatch paths are not W.x (quant_kernels_omp.c
    :199-209, 1647-1758 and 1778-1812); the fixture keeps that evidence."""
    n, k, _ = RO["shape"]
    exact = O.gemv(RO[f"gemv_w_{qt}"], qt, RO[f"gemv_x_{qt}"], n, k)[0]
    assert O.rel_l2(RO[f"gemv_ref_dispatch_{qt}"], exact) > 0.05


@pytest.mark.parametrize("qt", sorted(F.BLOCK), ids=lambda q: F.NAMES[q])
def test_quantize_roundtrip_is_a_valid_encoding(qt):
    rng = np.random.default_rng(qt)
    x = (rng.standard_normal(1024) * 0.02).astype(np.float32)
    raw = F.quantize(qt, x)
    assert raw.size == F.row_bytes(qt, 1024)
    back = F.dequantize(qt, raw, 1024)
    assert O.rel_l2(back, x) < 0.2


@pytest.mark.parametrize("tag", ["32_4_64_37", "16_2_256_200"])
def test_gqa_reference_output_is_modelled_and_deviates(tag):
    """gqa_attention_decode of the reference (gqa_attention.c:93) evaluates exp with a
    reversed polynomial (gqa_attention.c:32-48): the oracle's model of that quirk
    reproduces the reference's output, and the true softmax attention differs from it.
    The GPU kernels are checked against the true attention (oracle.ops.gqa_decode)."""
    nh, nkh, hd, sl = (int(t) for t in tag.split("_"))
    q, k, v = RO[f"gqa_q_{tag}"], RO[f"gqa_k_{tag}"], RO[f"gqa_v_{tag}"]
    assert O.rel_l2(RO[f"gqa_out_{tag}"], O.gqa_decode_reference_quirk(q, k, v, nh, nkh, hd)) < 1e-4
    assert O.rel_l2(RO[f"gqa_out_{tag}"], O.gqa_decode(q, k, v, nh, nkh, hd)) > 1e-2


def test_moe_oracle_matches_reference_c():
    ne, n_embd, n_ff, topk = (int(v) for v in RO["moe_dims"])
    g = {e: RO["moe_gate"][e] for e in range(ne)}
    u = {e: RO["moe_up"][e] for e in range(ne)}
    d = {e: RO["moe_down"][e] for e in range(ne)}
    got = O.moe_forward(g, u, d, (F.Q4_0, F.Q4_0, F.Q4_0), RO["moe_x"], n_ff, n_embd, RO["moe_idx"], RO["moe_w"])
    assert O.rel_l2(RO["moe_out"], got) < 1e-5


def test_router_tie_rule_and_renorm():
    lg = np.array([1.0, 3.0, 3.0, 0.5, 3.0], np.float32)
    idx, w = O.router_topk(lg, 2, renorm=True)
    assert list(idx) == [1, 2] and abs(float(w.sum()) - 1.0) < 1e-6


def test_ssm_oracle_matches_reference_c():
    B, N, inner, groups, ss, dtr = (int(v) for v in RO["ssm_dims"])
    interm, st = O.ssm_decode_step(RO["ssm_x"], RO["ssm_conv"], RO["ssm_a"], RO["ssm_dt"], RO["ssm_alpha"],
                                   RO["ssm_beta"], RO["ssm_state_in"], B, N, inner, groups, ss, dtr)
    assert O.rel_l2(RO["ssm_interm"], interm.reshape(-1)) < 1e-6
    assert O.rel_l2(RO["ssm_state_out"], st.reshape(-1)) < 1e-6
