"""Pins the numpy oracle to the reference's own outputs (golden fixtures).

The fixtures were produced by running NeuraTensor 4.0.4 itself
(tests/golden/make_golden.py).  Every oracle function used as the checker
of the CUDA path is compared here, in both arithmetic modes.
"""
import numpy as np
import pytest
import torch

from conftest import gget, golden_params, load_golden, unbits
from oracle import neuratensor_oracle as O


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_lif_scan_matches_reference_bit_exact(mode):
    d = load_golden(f"lif_{mode}.npz")
    x, beta, th, m0 = gget(d, "x"), gget(d, "beta"), gget(d, "theta"), gget(d, "mem0")
    spk, mem = O.lif_scan(x, m0, beta, th, mode)
    np.testing.assert_array_equal(spk, unbits(d["spikes_bits"], d["spikes_shape"]))
    np.testing.assert_array_equal(mem, gget(d, "mem_out"))
    spk0, mem0 = O.lif_scan(x, None, beta, th, mode)
    np.testing.assert_array_equal(spk0, unbits(d["spikes_fresh_bits"], d["spikes_shape"]))
    np.testing.assert_array_equal(mem0, gget(d, "mem_out_fresh"))
    s1, m1 = O.lif_step(x[:, 0], m0, beta, th, mode)
    np.testing.assert_array_equal(s1, gget(d, "step_spk"))
    np.testing.assert_array_equal(m1, gget(d, "step_mem"))


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_beta_sigmoid(mode):
    d = load_golden(f"lif_{mode}.npz")
    b = O.sigmoid(gget(d, "beta_logit"), mode)
    np.testing.assert_allclose(b, gget(d, "beta"), rtol=2e-7 if mode == "fp32" else 0, atol=0)


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_ssm_layer_matches_reference(mode):
    d = load_golden(f"ssm_{mode}.npz")
    p = golden_params(d)
    u, st0 = gget(d, "u"), gget(d, "st0")
    dt, Bm, Cm = O.ssm_projections(u, p, mode)
    np.testing.assert_allclose(dt, gget(d, "dt"), rtol=1e-6, atol=1e-7)
    np.testing.assert_array_equal(Bm, gget(d, "Bm"))
    np.testing.assert_array_equal(Cm, gget(d, "Cm"))
    tol = dict(rtol=1e-5, atol=1e-6) if mode == "fp32" else dict(rtol=0, atol=0)
    y, st = O.ssm_layer(u, p, st0, mode)
    np.testing.assert_allclose(y, gget(d, "y"), **tol)
    np.testing.assert_allclose(st, gget(d, "st"), **tol)
    y, st = O.ssm_layer(u, p, None, mode)
    np.testing.assert_allclose(y, gget(d, "y_fresh"), **tol)
    # split streaming == full sequence (the reference's own continuity test, tests/test_model.py:141-148)
    np.testing.assert_allclose(gget(d, "y_split"), gget(d, "y"), rtol=1e-5, atol=1e-4 if mode == "fp32" else 1e-2)


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_ssm_single_step(mode):
    """T=1 path (ssm.py:145-182).  In bf16, torch's CPU linear rounds the dt_proj
    bias add separately for tiny row counts, which can move dt by one bf16 ulp."""
    d = load_golden(f"ssm_{mode}.npz")
    p = golden_params(d)
    y, st = O.ssm_layer(gget(d, "u")[:, :1], p, gget(d, "st0"), mode)
    tol = dict(rtol=1e-5, atol=1e-6) if mode == "fp32" else dict(rtol=0, atol=2e-3)
    np.testing.assert_allclose(y, gget(d, "y1"), **tol)
    np.testing.assert_allclose(st, gget(d, "st1"), **tol)


def test_fused_lif_scan_matches_reference():
    d = load_golden("fused_op.npz")
    y, spk, mem, st = O.fused_lif_scan(gget(d, "x"), gget(d, "delta"), gget(d, "Bm"), gget(d, "Cm"), d["log_A"],
                                       d["D"], d["beta"], d["theta"], d["mem0"], d["st0"])
    np.testing.assert_array_equal(spk, unbits(d["spikes_bits"], d["spikes_shape"]))
    np.testing.assert_array_equal(mem, d["mem"])
    np.testing.assert_allclose(y, d["y"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(st, d["st"], rtol=1e-5, atol=1e-7)
    # channel-subset evaluation (used for full-size spot checks) agrees with the full one
    sel = np.array([1, 7, 30])
    ys, spks, mems, sts = O.fused_lif_scan(gget(d, "x"), gget(d, "delta"), gget(d, "Bm"), gget(d, "Cm"),
                                           d["log_A"], d["D"], d["beta"], d["theta"], d["mem0"], d["st0"],
                                           channels=sel)
    np.testing.assert_array_equal(ys, y[:, :, sel])
    np.testing.assert_array_equal(sts, st[:, sel])


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
@pytest.mark.parametrize("case", ["p10", "p25", "p50", "p70", "exact50", "none"])
def test_sparse_out_proj_matches_reference(mode, case):
    d = load_golden(f"sparse_out_{mode}.npz")
    o = gget(d, f"{case}_o")
    s = unbits(d[f"{case}_spikes_bits"], d[f"{case}_spikes_shape"])
    out = O.sparse_out_proj(o, s, gget(d, "W"), mode)
    ref = gget(d, f"{case}_out")
    if mode == "fp32":
        np.testing.assert_allclose(out, ref, rtol=1e-5, atol=2e-6)
    else:
        np.testing.assert_array_equal(out, ref)
    active = s.any(-1)
    assert np.all(ref[~active] == 0) or 2 * active.sum() > active.size


def test_block_forward_matches_reference():
    d = load_golden("block_fp32.npz")
    p = golden_params(d)
    x = d["x"]
    o1, s1, m1 = O.block_forward(x[:, :18], p, None, "fp32")
    o2, s2, m2 = O.block_forward(x[:, 18:], p, s1, "fp32")
    np.testing.assert_allclose(o1, d["out1"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(o2, d["out2"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(s1.membrane, d["mem1"], rtol=1e-5, atol=1e-6)   # h differs by GEMM order only
    np.testing.assert_allclose(s2.ssm_state, d["st2"], rtol=1e-5, atol=1e-7)
    assert m1["spike_rate"] == pytest.approx(float(d["rate1"]), abs=1e-9)
    assert m2["spike_rate"] == pytest.approx(float(d["rate2"]), abs=1e-9)


def test_attention_matches_reference():
    d = load_golden("attn_fp32.npz")
    p = golden_params(d)
    for k in ("long", "short"):
        y = O.attention(d[f"x_{k}"], p, n_heads=4, window=8, mode="fp32")
        np.testing.assert_allclose(y, d[f"y_{k}"], rtol=1e-4, atol=1e-5)


def _seeded_params(preset, seed):
    from neuratensor_b200 import NeuraTensorModel, get_preset
    torch.manual_seed(seed)
    m = NeuraTensorModel(get_preset(preset))
    return m, O.params_from_state_dict(m.state_dict())


def test_seeded_init_equals_reference_pico():
    d = load_golden("pico_fp32.npz")
    m, _ = _seeded_params("pico", 0)
    sd = m.state_dict()
    assert list(sd.keys()) == list(d["param_names"])
    for k, s, a in zip(d["param_names"], d["param_sum"], d["param_abs"]):
        assert float(sd[k].double().sum()) == pytest.approx(float(s), rel=1e-12, abs=1e-12), k
        assert float(sd[k].double().abs().sum()) == pytest.approx(float(a), rel=1e-12, abs=1e-12), k
    assert np.array_equal(torch.randint(0, 32000, (1, 64)).numpy(), d["ids"])


def test_pico_model_oracle_matches_reference():
    d = load_golden("pico_fp32.npz")
    _, p = _seeded_params("pico", 0)
    cfg = O.OracleConfig(vocab_size=32000, d_model=96, n_layers=4, d_state=8, max_seq_len=512)
    cap = []
    rows = d["logits_row_idx"]
    logits, states, metrics = O.model_forward(d["ids"], p, cfg, None, "fp32", capture=cap)
    spk = np.stack([c["spikes"] for c in cap])
    ref_spk = unbits(d["spikes_bits"], d["spikes_shape"])
    assert (spk == ref_spk).mean() >= 0.9999
    np.testing.assert_allclose(logits[0, rows], d["logits_rows"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(logits[0].sum(-1), d["logit_sum"], rtol=1e-3, atol=1e-3)
    np.testing.assert_array_equal(logits[0].argmax(-1), d["logit_argmax"])
    np.testing.assert_allclose(metrics["per_layer_spike_rate"], d["per_layer_rate"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(np.stack([s.membrane for s in states]), d["membrane"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(np.stack([s.ssm_state for s in states]), d["ssm_state"], rtol=1e-4, atol=1e-7)


def _small_bf16(matmul):
    d = load_golden("small_bf16.npz")
    m, p = _seeded_params("small", 1)
    for k in p:   # the reference runs the model cast to bf16 (engine.py:66)
        p[k] = O.bf16(p[k])
    cfg = O.OracleConfig(vocab_size=32000, d_model=640, n_layers=12, d_state=32, max_seq_len=2048,
                         attn_every=6, attn_heads=10, attn_window=256)
    cap = []
    O.set_matmul(matmul)
    try:
        logits, states, metrics = O.model_forward(d["ids"], p, cfg, None, "bf16", capture=cap,
                                                  logits_rows=d["logits_row_idx"])
    finally:
        O.set_matmul("numpy")
    shape = d["spikes_shape"]
    agree = [(cap[0]["spikes"] == unbits(d["spikes0_bits"], shape)).mean(),
             (cap[11]["spikes"] == unbits(d["spikes11_bits"], shape)).mean()]
    return d, logits, metrics, agree, cap


def test_small_bf16_oracle_matches_reference():
    """Small preset in bf16 (12 layers, 2 attention layers, T=320 > window).  With
    the reference's own CPU kernels for the GEMMs, rsqrt and attention core (the
    ops whose CPU rounding is not plain IEEE float32), every other op being the
    oracle's, the oracle reproduces the reference bit for bit."""
    d, logits, metrics, agree, cap = _small_bf16("torch")
    assert agree == [1.0, 1.0], agree
    for i, c in enumerate(cap):
        np.testing.assert_array_equal(c["spikes"].sum(-1), d["row_counts"][i])
    np.testing.assert_array_equal(logits[0], gget(d, "logits_rows"))
    assert metrics["per_layer_spike_rate"] == list(d["per_layer_rate"])


def test_small_bf16_is_chaotic_under_gemm_rounding():
    """The random-init model in bf16 amplifies one-ulp GEMM differences: with
    float32-BLAS products (about 1e-4 of in_proj outputs one bf16 ulp away from
    the reference's), layer 0 still agrees on >= 99.99% of spikes but deep layers
    drift.  Model-level bf16 parity is therefore checked layer by layer (each
    block fed the same input) in the GPU tests."""
    d, logits, metrics, agree, cap = _small_bf16("numpy")
    assert agree[0] >= 0.9999
    assert agree[1] < 0.995   # documents the amplification; not a property of any kernel here
    np.testing.assert_allclose(metrics["per_layer_spike_rate"], d["per_layer_rate"], rtol=5e-2)
