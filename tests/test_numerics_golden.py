"""The numerics oracle reproduces the reference's own numpy checks (CPU only).

tests/golden/numerics.npz holds inputs and outputs of the reference's numpy code,
executed unchanged from its example scripts by tests/golden/make_numerics_golden.py:
  benchmark_rmsnorm.py:115-116, benchmark_sdpa.py:198-208 (attention_ref),
  showcase_attention.py:150-153, qwen_megakernel.py:308-342 (rmsnorm_np, rope_np,
  full_decode_np) and :358-364 (the KV-cache pre-fill).
The reference computes in fp32 and the oracle in fp64, so agreement is to fp32
rounding (rtol 1e-5), the bar BASELINE sets for fp32 RMSNorm.
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import numerics as orc

G = np.load(Path(__file__).parent / "golden" / "numerics.npz")
RT, AT = 1e-5, 1e-6


def test_rmsnorm_matches_reference_check():
    got = orc.rmsnorm(G["rms_X"], G["rms_W"], float(G["rms_eps"]))
    np.testing.assert_allclose(got, G["rms_expected"], rtol=RT, atol=AT)


def test_rmsnorm_fp32_formula_matches_reference_check():
    got = orc.rmsnorm_fp32(G["rms_X"], G["rms_W"], float(G["rms_eps"]))
    np.testing.assert_array_equal(got, G["rms_expected"])


@pytest.mark.parametrize("qkey,okey", [("gqa_Q", "gqa_O"), ("gqa_Qpeak", "gqa_Opeak")])
def test_gqa_attention_matches_attention_ref(qkey, okey):
    """attention_ref: [T, Hq, D] queries, [Hkv, S, D] keys / values, no scale, kvh = qh // QMUL."""
    q, k, v = G[qkey], G["gqa_K"], G["gqa_V"]
    got = orc.sdpa(q.transpose(1, 0, 2)[None], k[None], v[None], 1.0)[0].transpose(1, 0, 2)
    np.testing.assert_allclose(got, G[okey], rtol=RT, atol=AT)


def test_gqa_peaked_case_is_peaked():
    """The peaked fixture really concentrates the softmax (max weight near 1 on some rows)."""
    q, k = G["gqa_Qpeak"], G["gqa_K"]
    s = np.einsum("thd,gsd->thgs", q.astype(np.float64), k.astype(np.float64))
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    assert p.max() > 0.5


def test_fa_matches_showcase_check():
    q, k, v = G["fa_Q"], G["fa_K"], G["fa_V"]
    got = orc.sdpa(q[None, None], k[None, None], v[None, None], 1 / np.sqrt(q.shape[1]))[0, 0]
    np.testing.assert_allclose(got, G["fa_O"], rtol=RT, atol=AT)


def test_rope_matches_rope_np():
    np.testing.assert_allclose(orc.rope(G["rope_x"], G["qwen_cos_pos"], G["qwen_sin_pos"]),
                               G["rope_out"], rtol=RT, atol=AT)


def _qwen():
    H, INTER, QH, KVH, HD, CL = (int(v) for v in G["qwen_shape"])
    w = {k[5:]: G[k] for k in G.files if k.startswith("qwen_")}
    return H, INTER, QH, KVH, HD, CL, w


def test_qwen_decode_f32_matches_full_decode_np():
    H, INTER, QH, KVH, HD, CL, w = _qwen()
    got = orc.qwen_decode_f32(w["x"], w["w_in_norm"], w["Wq"], w["Wk"], w["Wv"], w["w_q_norm"],
                              w["w_k_norm"], w["cos_pos"], w["sin_pos"], w["kc_filled"],
                              w["vc_filled"], w["Wo"], w["w_post_norm"], w["Wg"], w["Wu"],
                              w["Wd"], QH, KVH, 1e-6)
    np.testing.assert_allclose(got, w["out"], rtol=RT, atol=AT)


def test_batched_decode_layer_matches_full_decode_np():
    """The batched oracle the bf16 decode kernels are checked against, with the Qwen3
    head-norm switched on and the reference's weights packed into its [in, out] layout."""
    H, INTER, QH, KVH, HD, CL, w = _qwen()
    wd = {"w_in_norm": w["w_in_norm"], "w_post_norm": w["w_post_norm"],
          "w_qkv": np.concatenate([w["Wq"].T, w["Wk"].T, w["Wv"].T], axis=1),
          "w_o": w["Wo"].T, "w_gate_up": np.concatenate([w["Wg"].T, w["Wu"].T], axis=1),
          "w_down": w["Wd"].T}
    out, q, k, v = orc.decode_layer(w["x"][None], wd, w["k_cache"][None], w["v_cache"][None],
                                    w["cos_pos"], w["sin_pos"], CL, QH, KVH, HD, 1e-6,
                                    q_norm=w["w_q_norm"], k_norm=w["w_k_norm"])
    np.testing.assert_allclose(out[0], w["out"], rtol=RT, atol=AT)
    # the new key / value are the reference host's cache pre-fill (qwen_megakernel.py:358-364)
    np.testing.assert_allclose(k[0], w["kc_filled"][:, CL], rtol=RT, atol=AT)
    np.testing.assert_allclose(v[0], w["vc_filled"][:, CL], rtol=RT, atol=AT)
