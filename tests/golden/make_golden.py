"""Generate the golden fixtures in this folder by running the reference itself.

Test infrastructure, not product code.  It imports the reference package
(NeuraTensor 4.0.4, pure PyTorch) from the path given by ``--reference``
(default ``$NEURATENSOR_REFERENCE``) with telemetry off, drives the
hot-path functions on seeded inputs and writes small ``.npz`` fixtures:

  lif_{fp32,bf16}.npz      neuratensor/core/snn.py:64-75,167-182,260-262
  ssm_{fp32,bf16}.npz      neuratensor/core/ssm.py:34-43,106-139,145-221,313-349
  fused_op.npz             snn.py:167-182 + ssm.py:106-139,184-221 (LIF feeding the scan)
  sparse_out_{fp32,bf16}.npz  neuratensor/core/fused.py:149-165
  block_fp32.npz           neuratensor/core/fused.py:101-147
  pico_fp32.npz            neuratensor/core/model.py:240-293 (pico preset, seed 0)
  pico_stream.npz          split-vs-full streaming and T=1 decode steps
  small_bf16.npz           small preset through InferenceEngine.run in bf16 (seed 1)
  attn_fp32.npz            neuratensor/core/model.py:88-181

Run from the repository root:
    NEURATENSOR_TELEMETRY=0 python tests/golden/make_golden.py --reference <path>

bf16 tensors are stored as their raw uint16 bit patterns (key suffix ``_bf16``).
Spike tensors are stored bit-packed (``np.packbits`` over the last axis, key
suffix ``_bits``) together with their shape.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

OUT = os.path.dirname(os.path.abspath(__file__))


def _np(t):
    import torch
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def _bits(t):
    a = (t.detach().cpu().float().numpy() != 0)
    return np.packbits(a, axis=-1), np.array(a.shape, dtype=np.int64)


def _param_sums(model):
    """Per-parameter float64 checksums of a state_dict (pins the seeded init)."""
    names, sums, abss, heads = [], [], [], []
    for k, v in model.state_dict().items():
        f = v.detach().cpu().double().reshape(-1)
        names.append(k)
        sums.append(float(f.sum()))
        abss.append(float(f.abs().sum()))
        h = np.zeros(4)
        h[: min(4, f.numel())] = f[:4].numpy()
        heads.append(h)
    return dict(param_names=np.array(names), param_sum=np.array(sums),
                param_abs=np.array(abss), param_head=np.stack(heads))


def _logit_stats(logits):
    import torch
    f = logits.detach().float()
    return dict(logit_sum=f.sum(-1).double().numpy(),
                logit_sq=(f.double() ** 2).sum(-1).numpy(),
                logit_max=f.max(-1).values.numpy(),
                logit_argmax=f.argmax(-1).numpy().astype(np.int64))


def gen_lif(nt, torch):
    from neuratensor.core import snn
    for dt_name, dtype in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        g = torch.Generator().manual_seed(11)
        B, T, C = 3, 70, 37
        x = (torch.randn(B, T, C, generator=g) * 0.8 + 0.3).to(dtype)
        beta_logit = torch.logit(torch.rand(C, generator=g) * 0.19 + 0.80).to(dtype)
        beta = torch.sigmoid(beta_logit)
        scales = torch.ones(C)
        scales[C // 3: 2 * (C // 3)] = 1.5
        scales[2 * (C // 3):] = 2.0
        theta = (1.0 * scales).to(dtype)
        mem0 = (torch.randn(B, C, generator=g) * 0.5).to(dtype)
        spk, mem = snn._lif_sequential_scan(x, mem0, beta, theta, 10.0)
        # fresh state (LIFLayer.forward zero-init, snn.py:286-287)
        spk0, mem_z = snn._lif_sequential_scan(x, torch.zeros(B, C, dtype=dtype), beta, theta, 10.0)
        # T=1 fast path (snn.py:64-75)
        s1, m1 = snn._lif_single_step(x[:, 0, :], mem0, beta, theta, 10.0)
        sb, shape = _bits(spk)
        sb0, _ = _bits(spk0)
        d = dict(x=x, beta_logit=beta_logit, beta=beta, theta=theta, mem0=mem0,
                 mem_out=mem, mem_out_fresh=mem_z, step_spk=s1, step_mem=m1)
        out = {}
        for k, v in d.items():
            out[k + ("_bf16" if v.dtype == torch.bfloat16 else "")] = _np(v)
        out.update(spikes_bits=sb, spikes_shape=shape, spikes_fresh_bits=sb0)
        np.savez_compressed(os.path.join(OUT, f"lif_{dt_name}.npz"), **out)


def gen_ssm(nt, torch):
    from neuratensor.core.ssm import SelectiveSSMLayer
    for dt_name, dtype in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        torch.manual_seed(21)
        d, N = 24, 16
        layer = SelectiveSSMLayer(d_model=d, d_state=N)
        with torch.no_grad():
            # give Δ a useful range (trained-like), and exercise the |A|<1e-6 limit
            # branch of _discretize (ssm.py:129-137) on channel 3, state 5
            layer.dt_proj.bias.copy_(torch.randn(d) * 0.5 - 1.5)
            layer.log_A[3, 5] = -20.0
            layer.log_A[7] += torch.randn(N) * 0.1   # non-HiPPO channel
            layer.D.copy_(torch.rand(d) + 0.5)
        layer = layer.to(dtype)
        g = torch.Generator().manual_seed(22)
        B, T = 2, 40
        u = (torch.rand(B, T, d, generator=g) < 0.2).to(dtype)
        st0 = (torch.randn(B, d, N, generator=g) * 0.1).to(dtype)
        with torch.no_grad():
            y, st = layer(u, st0)
            y_fresh, st_fresh = layer(u, None)
            Bm = layer.B_proj(u)
            Cm = layer.C_proj(u)
            dt = torch.nn.functional.softplus(layer.dt_proj(u))
            y1, st1 = layer(u[:, :1], st0)          # T=1 path (ssm.py:145-182)
            ya, sa = layer(u[:, :17], st0)          # split streaming
            yb, sb = layer(u[:, 17:], sa)
        out = {}
        tens = dict(u=u, st0=st0, y=y, st=st, y_fresh=y_fresh, st_fresh=st_fresh,
                    Bm=Bm, Cm=Cm, dt=dt, y1=y1, st1=st1, y_split=torch.cat([ya, yb], 1), st_split=sb)
        for k, v in tens.items():
            out[k + ("_bf16" if v.dtype == torch.bfloat16 else "")] = _np(v)
        for k, v in layer.state_dict().items():
            out["w_" + k.replace(".", "_") + ("_bf16" if v.dtype == torch.bfloat16 else "")] = _np(v)
        np.savez_compressed(os.path.join(OUT, f"ssm_{dt_name}.npz"), **out)


def gen_fused_op(nt, torch):
    """LIF feeding the selective scan with given Δ/B/C (the standalone fused op)."""
    from neuratensor.core import snn
    from neuratensor.core.ssm import SelectiveSSMLayer
    g = torch.Generator().manual_seed(31)
    B, L, D, N = 2, 96, 40, 16
    x = torch.randn(B, L, D, generator=g).bfloat16()
    delta = torch.nn.functional.softplus(torch.randn(B, L, D, generator=g) - 2.0).bfloat16()
    Bm = (torch.randn(B, L, N, generator=g) / N ** 0.5).bfloat16()
    Cm = (torch.randn(B, L, N, generator=g) / N ** 0.5).bfloat16()
    beta = torch.rand(D, generator=g) * 0.19 + 0.80
    theta = torch.ones(D)
    mem0 = torch.randn(B, D, generator=g) * 0.5
    st0 = torch.randn(B, D, N, generator=g) * 0.1
    Dskip = torch.rand(D, generator=g) + 0.5
    layer = SelectiveSSMLayer(d_model=D, d_state=N)   # log_A = log(n+1) -> A = -(n+1)
    with torch.no_grad():
        spk, mem = snn._lif_sequential_scan(x.float(), mem0, beta, theta, 10.0)
        A_bar, B_bar = layer._discretize(delta.float(), Bm.float())
        y, st = layer._scan_sequential(spk, A_bar, B_bar, Cm.float(), Dskip, st0)
    sbits, shape = _bits(spk)
    np.savez_compressed(
        os.path.join(OUT, "fused_op.npz"),
        x_bf16=_np(x), delta_bf16=_np(delta), Bm_bf16=_np(Bm), Cm_bf16=_np(Cm),
        beta=_np(beta), theta=_np(theta), mem0=_np(mem0), st0=_np(st0), D=_np(Dskip),
        log_A=_np(layer.log_A), y=_np(y), st=_np(st), mem=_np(mem),
        spikes_bits=sbits, spikes_shape=shape)


def gen_sparse_out(nt, torch):
    from neuratensor.core.fused import FusedSpikeBlock
    for dt_name, dtype in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        torch.manual_seed(41)
        blk = FusedSpikeBlock(d_model=32, d_state=4, expand=2).to(dtype).eval()
        g = torch.Generator().manual_seed(42)
        B, T, di = 2, 40, 64
        out = {"W" + ("_bf16" if dtype == torch.bfloat16 else ""): _np(blk.out_proj.weight)}
        cases = {"p10": 0.10, "p25": 0.25, "p50": 0.50, "p70": 0.70}
        for name, p in list(cases.items()) + [("exact50", None), ("none", 0.0)]:
            o = torch.randn(B, T, di, generator=g).to(dtype)
            if name == "exact50":
                act = torch.zeros(B * T, dtype=torch.bool)
                act[torch.randperm(B * T, generator=g)[: B * T // 2]] = True
                act = act.view(B, T)
            else:
                act = torch.rand(B, T, generator=g) < p
            spk = (torch.rand(B, T, di, generator=g) < 0.2) & act[..., None]
            # rows flagged active must really have a spike
            first = torch.zeros(B, T, di, dtype=torch.bool)
            first[..., 0] = True
            spk = spk | (first & act[..., None])
            spk = spk.to(dtype)
            with torch.no_grad():
                res = blk._sparse_out_proj(o, spk)
            sfx = "_bf16" if dtype == torch.bfloat16 else ""
            out[f"{name}_o{sfx}"] = _np(o)
            b, shape = _bits(spk)
            out[f"{name}_spikes_bits"] = b
            out[f"{name}_spikes_shape"] = shape
            out[f"{name}_out{sfx}"] = _np(res)
        np.savez_compressed(os.path.join(OUT, f"sparse_out_{dt_name}.npz"), **out)


def gen_block(nt, torch):
    from neuratensor.core.fused import FusedSpikeBlock, BlockState
    torch.manual_seed(51)
    blk = FusedSpikeBlock(d_model=24, d_state=8, expand=2).eval()
    with torch.no_grad():
        blk.ssm.dt_proj.bias.copy_(torch.randn(48) * 0.5 - 1.5)
        blk.norm.weight.copy_(torch.rand(24) + 0.5)
    g = torch.Generator().manual_seed(52)
    x = torch.randn(2, 30, 24, generator=g) * 1.5
    with torch.no_grad():
        o1, s1, m1 = blk(x[:, :18])
        o2, s2, m2 = blk(x[:, 18:], s1)
        of, sf, mf = blk(x)
    out = dict(x=_np(x), out1=_np(o1), out2=_np(o2), out_full=_np(of),
               mem1=_np(s1.membrane), st1=_np(s1.ssm_state), mem2=_np(s2.membrane), st2=_np(s2.ssm_state),
               rate1=np.array(m1["spike_rate"]), rate2=np.array(m2["spike_rate"]),
               mean_beta=np.array(m1["mean_beta"]))
    for k, v in blk.state_dict().items():
        out["w_" + k.replace(".", "_")] = _np(v)
    np.savez_compressed(os.path.join(OUT, "block_fp32.npz"), **out)


def _capture_model(model, torch):
    """Forward hooks that record per-block spikes/states and block-0 internals."""
    rec = {"spikes": [], "h0": None}
    hooks = []
    for i, blk in enumerate(model.blocks):
        def snn_hook(mod, inp, outp, i=i):
            rec["spikes"].append(outp[0].detach().clone())
            if i == 0:
                rec["h0"] = inp[0].detach().clone()
        hooks.append(blk.snn.register_forward_hook(snn_hook))
    return rec, hooks


def gen_pico(nt, torch):
    from neuratensor import NeuraTensorModel, get_preset
    torch.manual_seed(0)
    model = NeuraTensorModel(get_preset("pico")).eval()
    ids = torch.randint(0, 32000, (1, 64))
    rec, hooks = _capture_model(model, torch)
    with torch.no_grad():
        logits, states, metrics = model(ids)
    for h in hooks:
        h.remove()
    spk = torch.stack(rec["spikes"])              # [L, B, T, di]
    sb, shape = _bits(spk)
    out = dict(ids=ids.numpy().astype(np.int64), spikes_bits=sb, spikes_shape=shape,
               membrane=np.stack([_np(s.membrane) for s in states]),
               ssm_state=np.stack([_np(s.ssm_state) for s in states]),
               per_layer_rate=np.array(metrics["per_layer_spike_rate"]),
               spike_rate=np.array(metrics["spike_rate"]),
               sparsity=np.array(metrics["estimated_sparsity_pct"]),
               logits_rows=_np(logits[0, [0, 31, 63]]), logits_row_idx=np.array([0, 31, 63]),
               h0=_np(rec["h0"]))
    out.update(_logit_stats(logits[0]))
    out.update(_param_sums(model))
    np.savez_compressed(os.path.join(OUT, "pico_fp32.npz"), **out)

    # streaming: 40 + 24 split with carried state, then 3 single-token steps
    with torch.no_grad():
        la, sa, _ = model(ids[:, :40])
        lb, sb_, mb = model(ids[:, 40:], sa)
        steps = []
        st = sb_
        nxt = ids[:, -1:]
        dec_ids = []
        for k in range(3):
            nxt = (nxt * 7 + 13 + k) % 32000
            dec_ids.append(int(nxt))
            lg, st, _ = model(nxt, st)
            steps.append(lg[0, 0])
    out = dict(split_rows=_np(torch.stack([la[0, 39], lb[0, 0], lb[0, 23]])),
               split_membrane=np.stack([_np(s.membrane) for s in sb_]),
               split_ssm_state=np.stack([_np(s.ssm_state) for s in sb_]),
               split_rates=np.array(mb["per_layer_spike_rate"]),
               decode_ids=np.array(dec_ids), decode_rows=_np(torch.stack(steps)),
               decode_membrane=np.stack([_np(s.membrane) for s in st]),
               decode_ssm_state=np.stack([_np(s.ssm_state) for s in st]))
    np.savez_compressed(os.path.join(OUT, "pico_stream.npz"), **out)


def gen_small_bf16(nt, torch):
    from neuratensor import NeuraTensorModel, get_preset, InferenceEngine
    torch.manual_seed(1)
    model = NeuraTensorModel(get_preset("small"))
    sums = _param_sums(model)
    ids = torch.randint(0, 32000, (1, 320))
    eng = InferenceEngine(model, device="cpu", dtype=torch.bfloat16)
    rec, hooks = _capture_model(eng.model, torch)
    res = eng.run(ids, reset_state=True)
    for h in hooks:
        h.remove()
    spk = torch.stack(rec["spikes"])               # [12, 1, 320, 1280]
    b0, shape0 = _bits(spk[0])
    b11, _ = _bits(spk[11])
    rows = [0, 100, 255, 256, 319]
    out = dict(ids=ids.numpy().astype(np.int64),
               spikes0_bits=b0, spikes11_bits=b11, spikes_shape=shape0,
               row_counts=spk.float().sum(-1).numpy().astype(np.int64),   # [12,1,320]
               per_layer_rate=np.array(res.metrics["per_layer_spike_rate"]),
               spike_rate=np.array(res.metrics["spike_rate"]),
               logits_rows_bf16=_np(res.logits[0, rows]), logits_row_idx=np.array(rows),
               membrane0_bf16=_np(res.states[0].membrane),
               ssm_state0_bf16=_np(res.states[0].ssm_state),
               membrane11_bf16=_np(res.states[11].membrane),
               h0_bf16=_np(rec["h0"][0, :64]))
    out.update(_logit_stats(res.logits[0]))
    out.update(sums)
    np.savez_compressed(os.path.join(OUT, "small_bf16.npz"), **out)


def gen_attn(nt, torch):
    from neuratensor.core.model import SlidingWindowAttention
    torch.manual_seed(61)
    attn = SlidingWindowAttention(d_model=32, n_heads=4, window=8).eval()
    g = torch.Generator().manual_seed(62)
    x_long = torch.randn(2, 20, 32, generator=g)
    x_short = torch.randn(2, 6, 32, generator=g)
    with torch.no_grad():
        y_long = attn(x_long)
        y_short = attn(x_short)
    out = dict(x_long=_np(x_long), y_long=_np(y_long), x_short=_np(x_short), y_short=_np(y_short))
    for k, v in attn.state_dict().items():
        out["w_" + k.replace(".", "_")] = _np(v)
    np.savez_compressed(os.path.join(OUT, "attn_fp32.npz"), **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("NEURATENSOR_REFERENCE", ""))
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    if not args.reference or not os.path.isdir(args.reference):
        sys.exit("pass --reference <path to the NeuraTensor 4.0.4 source tree>")
    os.environ["NEURATENSOR_TELEMETRY"] = "0"
    sys.path.insert(0, args.reference)
    import torch
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    import neuratensor as nt
    assert nt.__version__ == "4.0.4", nt.__version__
    gens = dict(lif=gen_lif, ssm=gen_ssm, fused_op=gen_fused_op, sparse_out=gen_sparse_out,
                block=gen_block, pico=gen_pico, small=gen_small_bf16, attn=gen_attn)
    for name, fn in gens.items():
        if args.only and name not in args.only.split(","):
            continue
        fn(nt, torch)
        print("wrote", name)


if __name__ == "__main__":
    main()
