"""Pin the CPU oracle to the reference's own outputs (golden fixtures).

The fixtures were produced by running the reference implementation on the
seeded inputs of ``tests/golden/cases.py`` (``tests/golden/make_golden.py``).
Byte work must be bit-exact; the floating-point restatements use the same
torch ops in the same order as the reference, so they must agree to
round-off (tolerances written per test).
"""

import numpy as np
import pytest
import torch

import cases
from oracle import attention as oa
from oracle import quant as oq
from oracle.model import OracleModel
from kshipra_b200.config import QWEN25_05B, TINY_LLAMA
from kshipra_b200.weights import synthetic_state_dict, weights_checksum


def test_oracle_quant_bit_exact(golden):
    g = golden("quant.npz")
    for name, w, scheme, gs in cases.quant_cases():
        wn = w.numpy()
        if scheme == "int8":
            p, s = oq.quantize_int8_per_channel(wn)
        else:
            p, s, _ = oq.quantize_int4_per_group(wn, gs)
        np.testing.assert_array_equal(p, g[f"{name}/payload"], err_msg=name)
        np.testing.assert_array_equal(s.view(np.uint16), g[f"{name}/scales"].view(np.uint16),
                                      err_msg=name)


def test_oracle_quant_edge_semantics():
    # scale underflow: +x -> +127, 0 -> 0 (NaN), -x -> -127; int4 gives -8 for -x
    w = np.zeros((1, 128), np.float32)
    w[0, :3] = [1e-7, 0.0, -2e-7]
    p, s = oq.quantize_int8_per_channel(w)
    assert s[0] == 0 and list(p[0, :3]) == [127, 0, -127]
    p4, s4, _ = oq.quantize_int4_per_group(w, 128)
    q = oq.unpack_int4(p4)
    assert list(q[0, :3]) == [7, 0, -8]
    with pytest.raises(ValueError):
        oq.quantize_int8_per_channel(np.array([[1.0, np.nan]], np.float32))
    with pytest.raises(ValueError):
        oq.quantize_int4_per_group(np.ones((2, 4), np.float32), 3)


def test_oracle_attention_matches_reference(golden):
    g = golden("attention.npz")
    for c in cases.attention_cases():
        q, kp, vp, bt = cases.attention_inputs(c)
        out = oa.chunked_attention(q, kp, vp, bt, c["P"], c["C"], c["B"]).numpy()
        np.testing.assert_allclose(out, g[c["name"]], rtol=0, atol=1e-6, err_msg=c["name"])
        if c["name"] + "/monolithic" in g:
            ref = g[c["name"] + "/monolithic"]
            rel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
            assert rel < 1e-5, (c["name"], rel)   # test_chunked_prefill.py:50-52
    q, kp, vp, bt, P, C, B = cases.mask_kat_inputs()
    np.testing.assert_allclose(oa.chunked_attention(q, kp, vp, bt, P, C, B).numpy(),
                               g["mask_kat"], atol=1e-6)


@pytest.mark.parametrize("scheme", ["int8", "int4", "none"])
def test_oracle_tiny_model_matches_reference(golden, scheme):
    g = golden("model_tiny.npz")
    sd = synthetic_state_dict(TINY_LLAMA, seed=0)
    assert weights_checksum(sd) == pytest.approx(float(g["weights_checksum"]), rel=1e-12)
    om = OracleModel(TINY_LLAMA, sd, None if scheme == "none" else scheme)
    toks, logs = om.generate(g["prompt"].tolist(), 16, block_size=16, prefill_chunk=16,
                             return_logits=True)
    assert toks == g[f"{scheme}/tokens"].tolist()
    L = torch.stack(logs).numpy()
    ref = g[f"{scheme}/logits"]
    assert np.abs(L - ref).max() <= 1e-5 * np.abs(ref).max()
    # chunked prefill == one-shot prefill of the reference's own generate
    assert g[f"{scheme}/tokens_oneshot"].tolist() == toks


def test_oracle_05b_prefill_matches_reference(golden):
    """0.5B shape, INT8: chunked prefill (4 x 128) + 2 decode tokens."""
    g = golden("model_qwen05b.npz")
    sd = synthetic_state_dict(QWEN25_05B, seed=0)
    assert weights_checksum(sd) == pytest.approx(float(g["weights_checksum"]), rel=1e-12)
    om = OracleModel(QWEN25_05B, sd, "int8")
    toks, logs = om.generate(g["prompt"].tolist(), 3, block_size=16, prefill_chunk=128,
                             return_logits=True)
    assert toks == g["int8/tokens"][:3].tolist()
    ref = g["int8/logits0"]
    assert np.abs(logs[0].numpy() - ref).max() <= 1e-5 * np.abs(ref).max()


def test_oracle_llama8b_l2_matches_reference(golden):
    """Llama-3-8B shape cut to two layers, INT4: one short batch prompt, two tokens."""
    g = golden("model_llama8b_l2.npz")
    cfg = cases.llama8b_l2()
    sd = synthetic_state_dict(cfg, seed=0)
    assert weights_checksum(sd) == pytest.approx(float(g["weights_checksum"]), rel=1e-12)
    om = OracleModel(cfg, sd, "int4")
    del sd
    p = cases.llama8b_batch_prompts(cfg.vocab)[4]
    assert om.generate(p, 2, block_size=16) == g["int4/batch4/tokens"][:2].tolist()


def test_oracle_cb_request_matches_reference(golden):
    """A shortened config-3 request (system prefix + trace suffix), INT4 0.5B, two tokens."""
    g = golden("model_cb_requests.npz")
    sd = synthetic_state_dict(QWEN25_05B, seed=0)
    om = OracleModel(QWEN25_05B, sd, "int4")
    p = cases.cb_requests(QWEN25_05B.vocab)[1]
    assert om.generate(p, 2, block_size=16) == g["req1/tokens"][:2].tolist()
