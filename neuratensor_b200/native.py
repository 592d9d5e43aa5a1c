"""ctypes binding of libneuratensor_native.so (the C ABI in include/neuratensor_native.h).

Each wrapper takes torch CUDA tensors, checks them, allocates the outputs
and the workspace through torch's caching allocator and calls the C entry
point on the current CUDA stream.  There is no fallback: if the library is
missing or the tensors are not on an sm_100 GPU, the call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional, Tuple

import torch
from torch import Tensor

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libneuratensor_native.so")

NT_F32, NT_BF16, NT_U8 = 0, 1, 2
_DT = {torch.float32: NT_F32, torch.bfloat16: NT_BF16}
_STATUS = {1: "bad argument", 2: "unsupported dtype", 3: "unsupported GPU", 4: "CUDA error",
           5: "device wait timed out", 6: "workspace too small"}


class NativeError(RuntimeError):
    """A libneuratensor_native call returned a non-zero status."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn}: {msg or _STATUS.get(status, 'error')} (status {status})")
        self.status = status


_lib = None
_lock = threading.Lock()
_I64, _I32, _P = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p

_SIGS = {
    "nt_abi_version": ([], _I32),
    "nt_last_error": ([], ctypes.c_char_p),
    "nt_device_supported": ([_I32], _I32),
    "nt_get_error_flag": ([_I32, ctypes.POINTER(ctypes.c_uint), _I32], _I32),
    "nt_launch_count": ([], ctypes.c_ulonglong),
    "nt_bounded_wait_check": ([_I64, _P], _I32),
    "nt_lif_scan": ([_I32, _I64, _I64, _I64, _P, _I64, _I64, _P, _P, _P, _P, _P, _I64, _I64, _P, _P], _I32),
    "nt_selective_scan": ([_I32, _I32, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P], _I32),
    "nt_ssm_workspace_bytes": ([_I32, _I64, _I64, _I64, _I64], _I64),
    "nt_ssm_forward": ([_I32, _I32, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _P], _I32),
    "nt_sparse_out_proj_workspace_bytes": ([_I32, _I64, _I64, _I64], _I64),
    "nt_sparse_out_proj": ([_I32, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _I64, _P], _I32),
    "nt_rmsnorm_in_proj_workspace_bytes": ([_I32, _I64, _I64, _I64], _I64),
    "nt_rmsnorm_in_proj": ([_I32, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _I64, _P], _I32),
    "nt_noalloc_scratch_bytes": ([], ctypes.c_size_t),
    "nt_rmsnorm_in_proj_noalloc": ([_I32, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P], _I32),
    "nt_block_workspace_bytes": ([_I32, _I64, _I64, _I64, _I64, _I64], _I64),
    "nt_block_forward": ([_I32, _I32, _I64, _I64, _I64, _I64, _I64] + [_P] * 17 + [_I32, _P, _I64, _P], _I32),
    "nt_lif_ssm_fused": ([_I64, _I64, _I64, _I64] + [_P] * 14 + [_I32, _P, _P], _I32),
    "nt_window_attention": ([_I32, _I64, _I64, _I64, _I64, _I64, _P, _I64, _P, _P, _P, _I64, _P], _I32),
    "nt_embedding": ([_I32, _I64, _I64, _I64, _P, _P, _P, _P], _I32),
    "nt_greedy_tokens": ([_I32, _I64, _I64, _P, _I64, _P, _P, _P], _I32),
    "nt_attention_workspace_bytes": ([_I32, _I64, _I64, _I64], _I64),
    "nt_attention_forward": ([_I32, _I64, _I64, _I64, _I64, _I64] + [_P] * 8 + [_I64, _P], _I32),
    "nt_lm_head_workspace_bytes": ([_I32, _I64, _I64, _I64], _I64),
    "nt_lm_head": ([_I32, _I64, _I64, _I64, _P, _P, _P, _P, _P, _I64, _P], _I32),
}

EXPORTED = tuple(_SIGS)


def library_path() -> str:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load the shared library once (raises NativeError when it is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise NativeError("load", 4, f"{_LIB_PATH} is missing; build it with "
                                  "`python -m neuratensor_b200.build`")
            lib = ctypes.CDLL(_LIB_PATH)
            for name, (args, res) in _SIGS.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            _lib = lib
    return _lib


def _check(fn: str, rc: int) -> None:
    if rc != 0:
        msg = load().nt_last_error().decode(errors="replace")
        raise NativeError(fn, rc, msg)


def _p(t: Optional[Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(dev: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


_checked_devices = set()


def _require_cuda(*ts: Optional[Tensor]) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("neuratensor_b200 runs its hot path on CUDA (sm_100 / B200) only; "
                               f"got a tensor on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise RuntimeError("no CUDA tensor given")
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _checked_devices:
        _check("nt_device_supported", load().nt_device_supported(idx))
        _checked_devices.add(idx)
    return dev


def _dtype_code(t: Tensor) -> int:
    if t.dtype not in _DT:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float32 or bfloat16")
    return _DT[t.dtype]


def _workspace(nbytes: int, dev) -> Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=dev)


def _c(t: Optional[Tensor], dtype=None) -> Optional[Tensor]:
    if t is None:
        return None
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


# --------------------------------------------------------------------------- #
#  Entry points                                                                #
# --------------------------------------------------------------------------- #

def lif_scan(x: Tensor, beta: Tensor, threshold: Tensor, membrane: Optional[Tensor] = None,
             spike_count: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
    """LIFLayer.forward (snn.py:264-312): x [B,T,C] -> (spikes [B,T,C], membrane [B,C])."""
    dev = _require_cuda(x, beta, threshold, membrane)
    if x.dim() != 3:
        raise ValueError(f"x must be [B, T, C], got {tuple(x.shape)}")
    B, T, C = x.shape
    if x.stride(2) != 1:
        x = x.contiguous()
    dt = x.dtype
    beta, threshold = _c(beta, dt), _c(threshold, dt)
    if beta.numel() != C or threshold.numel() != C:
        raise ValueError("beta / threshold must have C elements")
    mem_in = None if membrane is None else _c(membrane, dt)
    if mem_in is not None and mem_in.shape != (B, C):
        raise ValueError(f"membrane must be [B, C] = {(B, C)}, got {tuple(mem_in.shape)}")
    spikes = torch.empty((B, T, C), dtype=dt, device=dev)
    mem_out = torch.empty((B, C), dtype=dt, device=dev)
    rc = load().nt_lif_scan(_dtype_code(x), B, T, C, _p(x), x.stride(0), x.stride(1), _p(beta), _p(threshold),
                            _p(mem_in), _p(mem_out), _p(spikes), spikes.stride(0), spikes.stride(1),
                            _p(spike_count), _stream(dev))
    _check("nt_lif_scan", rc)
    return spikes, mem_out


def selective_scan(u: Tensor, dt: Tensor, Bm: Tensor, Cm: Tensor, log_A: Tensor, D: Tensor,
                   state: Optional[Tensor] = None, gate: Optional[Tensor] = None,
                   state_dtype: Optional[torch.dtype] = None) -> Tuple[Tensor, Tensor]:
    """_discretize + _scan_sequential (ssm.py:106-139,184-221) -> (y [B,T,d], state [B,d,N])."""
    dev = _require_cuda(u, dt, Bm, Cm, log_A, D, state, gate)
    a = u.dtype
    B, T, d = u.shape
    N = log_A.shape[-1]
    sdt = state_dtype or (state.dtype if state is not None else a)
    u, dt, Bm, Cm, log_A, D = (_c(t, a) for t in (u, dt, Bm, Cm, log_A, D))
    gate = _c(gate, a)
    st_in = _c(state, sdt)
    y = torch.empty((B, T, d), dtype=a, device=dev)
    st_out = torch.empty((B, d, N), dtype=sdt, device=dev)
    rc = load().nt_selective_scan(_dtype_code(u), _DT[sdt], B, T, d, N, _p(u), _p(dt), _p(Bm), _p(Cm), _p(log_A),
                                  _p(D), _p(gate), _p(st_in), _p(st_out), _p(y), _stream(dev))
    _check("nt_selective_scan", rc)
    return y, st_out


def ssm_forward(u: Tensor, W_proj: Tensor, b_dt: Tensor, log_A: Tensor, D: Tensor,
                state: Optional[Tensor] = None, state_dtype: Optional[torch.dtype] = None) -> Tuple[Tensor, Tensor]:
    """SelectiveSSMLayer.forward (ssm.py:313-349) with the packed [W_dt; W_B; W_C] weight."""
    dev = _require_cuda(u, W_proj, b_dt, log_A, D, state)
    a = u.dtype
    B, T, d = u.shape
    N = log_A.shape[-1]
    sdt = state_dtype or (state.dtype if state is not None else a)
    u = _c(u)
    st_in = _c(state, sdt)
    y = torch.empty((B, T, d), dtype=a, device=dev)
    st_out = torch.empty((B, d, N), dtype=sdt, device=dev)
    L = load()
    nbytes = L.nt_ssm_workspace_bytes(_DT[a], B, T, d, N)
    ws = _workspace(nbytes, dev)
    rc = L.nt_ssm_forward(_DT[a], _DT[sdt], B, T, d, N, _p(u), _p(W_proj), _p(b_dt), _p(log_A), _p(D), _p(st_in),
                          _p(st_out), _p(y), _p(ws), nbytes, _stream(dev))
    _check("nt_ssm_forward", rc)
    return y, st_out


def sparse_out_proj(o: Tensor, spikes: Tensor, W: Tensor) -> Tuple[Tensor, Tensor]:
    """_sparse_out_proj (fused.py:149-165): returns (out, n_active as a device int64 tensor)."""
    dev = _require_cuda(o, spikes, W)
    a = o.dtype
    lead = o.shape[:-1]
    K = o.shape[-1]
    M = o.numel() // K
    Nout = W.shape[0]
    o2, s2, W2 = _c(o), _c(spikes, a), _c(W, a)
    out = torch.empty((*lead, Nout), dtype=a, device=dev)
    n_active = torch.empty((), dtype=torch.int64, device=dev)
    L = load()
    nbytes = L.nt_sparse_out_proj_workspace_bytes(_DT[a], M, K, Nout)
    ws = _workspace(nbytes, dev)
    rc = L.nt_sparse_out_proj(_DT[a], M, K, Nout, _p(o2), _p(s2), _p(W2), _p(out), _p(n_active), _p(ws), nbytes,
                              _stream(dev))
    _check("nt_sparse_out_proj", rc)
    return out, n_active


def rmsnorm_in_proj(x: Tensor, gamma: Tensor, W_in: Tensor) -> Tuple[Tensor, Tensor]:
    """norm + in_proj + chunk (fused.py:118-119): x [..., dm] -> (h, gate) [..., di]."""
    dev = _require_cuda(x, gamma, W_in)
    a = x.dtype
    dm = x.shape[-1]
    di = W_in.shape[0] // 2
    M = x.numel() // dm
    x2, g2, W2 = _c(x), _c(gamma, a), _c(W_in, a)
    h = torch.empty((*x.shape[:-1], di), dtype=a, device=dev)
    gate = torch.empty_like(h)
    L = load()
    nbytes = L.nt_rmsnorm_in_proj_workspace_bytes(_DT[a], M, dm, di)
    ws = _workspace(nbytes, dev)
    rc = L.nt_rmsnorm_in_proj(_DT[a], M, dm, di, _p(x2), _p(g2), _p(W2), _p(h), _p(gate), _p(ws), nbytes,
                              _stream(dev))
    _check("nt_rmsnorm_in_proj", rc)
    return h, gate


def rmsnorm_in_proj_noalloc(x: Tensor, gamma: Tensor, W_in: Tensor) -> Tuple[Tensor, Tensor]:
    """rmsnorm_in_proj without a workspace: for callers that cannot allocate device
    memory at call time; the library's own static scratch holds the normalised rows
    (at most nt_noalloc_scratch_bytes() of them).  Calls overlapping on the GPU race."""
    dev = _require_cuda(x, gamma, W_in)
    a = x.dtype
    dm = x.shape[-1]
    di = W_in.shape[0] // 2
    M = x.numel() // dm
    x2, g2, W2 = _c(x), _c(gamma, a), _c(W_in, a)
    h = torch.empty((*x.shape[:-1], di), dtype=a, device=dev)
    gate = torch.empty_like(h)
    rc = load().nt_rmsnorm_in_proj_noalloc(_DT[a], M, dm, di, _p(x2), _p(g2), _p(W2), _p(h), _p(gate), _stream(dev))
    _check("nt_rmsnorm_in_proj_noalloc", rc)
    return h, gate


def block_forward(x: Tensor, norm_w: Tensor, W_in: Tensor, beta: Tensor, threshold: Tensor, log_A: Tensor,
                  D: Tensor, W_proj: Tensor, b_dt: Tensor, W_out: Tensor, out_scale: Tensor,
                  membrane: Optional[Tensor], ssm_state: Optional[Tensor], spike_count: Tensor,
                  sparse: bool = True, state_dtype: Optional[torch.dtype] = None,
                  workspace: Optional[Tensor] = None) -> Tuple[Tensor, Tensor, Tensor]:
    """FusedSpikeBlock.forward (fused.py:101-147) -> (out, membrane, ssm_state).

    All weight tensors must already be contiguous and in x.dtype; spike_count
    is a device int64 scalar incremented by the block's spike count.
    """
    dev = x.device
    a = x.dtype
    B, T, dm = x.shape
    di = W_in.shape[0] // 2
    N = log_A.shape[-1]
    sdt = state_dtype or a
    x = x.contiguous()
    mem_in = None if membrane is None else _c(membrane, a)
    st_in = None if ssm_state is None else _c(ssm_state, sdt)
    out = torch.empty_like(x)
    mem_out = torch.empty((B, di), dtype=a, device=dev)
    st_out = torch.empty((B, di, N), dtype=sdt, device=dev)
    L = load()
    nbytes = L.nt_block_workspace_bytes(_DT[a], B, T, dm, di, N)
    ws = workspace if (workspace is not None and workspace.numel() >= nbytes) else _workspace(nbytes, dev)
    rc = L.nt_block_forward(_DT[a], _DT[sdt], B, T, dm, di, N, _p(x), _p(norm_w), _p(W_in), _p(beta), _p(threshold),
                            _p(log_A), _p(D), _p(W_proj), _p(b_dt), _p(W_out), _p(out_scale), _p(mem_in),
                            _p(mem_out), _p(st_in), _p(st_out), _p(out), _p(spike_count), 1 if sparse else 0,
                            _p(ws), ws.numel(), _stream(dev))
    _check("nt_block_forward", rc)
    return out, mem_out, st_out


def block_workspace_bytes(dtype: torch.dtype, B: int, T: int, dm: int, di: int, N: int) -> int:
    return int(load().nt_block_workspace_bytes(_DT[dtype], B, T, dm, di, N))


def lif_ssm_fused(x: Tensor, delta: Tensor, Bm: Tensor, Cm: Tensor, log_A: Tensor, Dskip: Tensor, beta: Tensor,
                  threshold: Tensor, membrane: Optional[Tensor] = None, state: Optional[Tensor] = None,
                  spike_dtype: Optional[torch.dtype] = torch.uint8, spike_count: Optional[Tensor] = None):
    """LIF spikes of x driving the selective scan with given dt/B/C (bf16 activations, fp32 state).

    Returns (y [B,L,d] bf16, spikes [B,L,d] or None, membrane [B,d] f32, state [B,d,N] f32).
    """
    dev = _require_cuda(x, delta, Bm, Cm, log_A, Dskip, beta, threshold, membrane, state)
    B, L_, d = x.shape
    N = log_A.shape[-1]
    bf = torch.bfloat16
    x, delta, Bm, Cm = (_c(t, bf) for t in (x, delta, Bm, Cm))
    log_A, Dskip, beta, threshold = (_c(t, torch.float32) for t in (log_A, Dskip, beta, threshold))
    mem_in = _c(membrane, torch.float32)
    st_in = _c(state, torch.float32)
    y = torch.empty((B, L_, d), dtype=bf, device=dev)
    spikes = None if spike_dtype is None else torch.empty((B, L_, d), dtype=spike_dtype, device=dev)
    sd = {torch.uint8: NT_U8, torch.bfloat16: NT_BF16, None: NT_U8}[spike_dtype]
    mem_out = torch.empty((B, d), dtype=torch.float32, device=dev)
    st_out = torch.empty((B, d, N), dtype=torch.float32, device=dev)
    rc = load().nt_lif_ssm_fused(B, L_, d, N, _p(x), _p(delta), _p(Bm), _p(Cm), _p(log_A), _p(Dskip), _p(beta),
                                 _p(threshold), _p(mem_in), _p(mem_out), _p(st_in), _p(st_out), _p(y), _p(spikes),
                                 sd, _p(spike_count), _stream(dev))
    _check("nt_lif_ssm_fused", rc)
    return y, spikes, mem_out, st_out


def window_attention(qkv: Tensor, n_heads: int, window: int, cos: Tensor, sin: Tensor) -> Tensor:
    """RoPE + sliding-window causal SDPA of SlidingWindowAttention.forward (model.py:159-178).

    qkv: [B, T, 3*d_model] bf16 (the qkv projection's output), head_dim =
    d_model / n_heads of 64 or 128; cos/sin: [T, head_dim] rotary tables;
    returns the attention output [B, T, d_model] (heads concatenated, as
    o_proj takes it)."""
    dev = _require_cuda(qkv, cos, sin)
    if qkv.dtype != torch.bfloat16:
        raise NativeError("nt_window_attention", 2, "bf16 only")
    if qkv.dim() != 3:
        raise ValueError(f"qkv must be [B, T, 3*d_model], got {tuple(qkv.shape)}")
    B, T, three_dm = qkv.shape
    dm = three_dm // 3
    hd = dm // n_heads if n_heads > 0 else 0
    if three_dm != 3 * dm or hd not in (64, 128) or dm != hd * n_heads:
        raise ValueError(f"qkv width {three_dm} does not split into {n_heads} heads of 64 or 128")
    if qkv.stride(2) != 1 or qkv.stride(0) != T * qkv.stride(1):
        qkv = qkv.contiguous()
    cos = cos[:T].to(torch.bfloat16).contiguous()
    sin = sin[:T].to(torch.bfloat16).contiguous()
    if cos.shape != (T, hd) or sin.shape != (T, hd):
        raise ValueError(f"cos/sin must hold at least T rows of {hd}")
    out = torch.empty((B, T, dm), dtype=torch.bfloat16, device=dev)
    rc = load().nt_window_attention(_dtype_code(qkv), B, T, n_heads, hd, int(window), _p(qkv), qkv.stride(1),
                                    _p(cos), _p(sin), _p(out), out.stride(1), _stream(dev))
    _check("nt_window_attention", rc)
    return out


def attention_forward(x: Tensor, norm_w: Tensor, W_qkv: Tensor, W_o: Tensor, n_heads: int, window: int,
                      cos: Tensor, sin: Tensor, workspace: Optional[Tensor] = None) -> Tensor:
    """SlidingWindowAttention.forward (model.py:148-181) in one call: RMSNorm, qkv
    projection, RoPE + windowed causal attention, o_proj + residual.  bf16, head_dim 64 or 128."""
    dev = _require_cuda(x, norm_w, W_qkv, W_o, cos, sin)
    if x.dtype != torch.bfloat16:
        raise NativeError("nt_attention_forward", 2, "bf16 only")
    B, T, dm = x.shape
    hd = dm // n_heads
    x = x.contiguous()
    nw, Wq, Wo = _c(norm_w, x.dtype), _c(W_qkv, x.dtype), _c(W_o, x.dtype)
    cos = cos[:T].to(torch.bfloat16).contiguous()
    sin = sin[:T].to(torch.bfloat16).contiguous()
    if cos.shape != (T, hd) or sin.shape != (T, hd):
        raise ValueError(f"cos/sin must hold at least T rows of {hd}")
    out = torch.empty_like(x)
    L = load()
    nbytes = L.nt_attention_workspace_bytes(_DT[x.dtype], B, T, dm)
    ws = workspace if (workspace is not None and workspace.numel() >= nbytes) else _workspace(nbytes, dev)
    rc = L.nt_attention_forward(_DT[x.dtype], B, T, dm, n_heads, int(window), _p(x), _p(nw), _p(Wq), _p(Wo),
                                _p(cos), _p(sin), _p(out), _p(ws), ws.numel(), _stream(dev))
    _check("nt_attention_forward", rc)
    return out


def greedy_tokens(logits: Tensor, u: Tensor, out: Optional[Tensor] = None) -> Tensor:
    """top_k = 1 sampling of generate (model.py:344-359): per row of logits [B, V],
    uniformly among the entries equal to the row maximum, chosen by u [B] in [0, 1).
    Returns int64 tokens [B, 1] (written into `out` when given)."""
    dev = _require_cuda(logits, u)
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be [B, V] with unit column stride")
    B, V = logits.shape
    u = _c(u, torch.float32)
    if out is None:
        out = torch.empty((B, 1), dtype=torch.int64, device=dev)
    rc = load().nt_greedy_tokens(_dtype_code(logits), B, V, _p(logits), logits.stride(0), _p(u), _p(out),
                                 _stream(dev))
    _check("nt_greedy_tokens", rc)
    return out


def embedding(ids: Tensor, W: Tensor) -> Tensor:
    """nn.Embedding lookup (model.py:258): ids [...] int64 -> [..., d_model] in W's dtype.
    An id outside [0, vocab) gives a zero row and a flag in the device error word."""
    dev = _require_cuda(ids, W)
    W = _c(W)
    ids = ids.to(torch.int64).contiguous()
    vocab, dm = W.shape
    out = torch.empty((*ids.shape, dm), dtype=W.dtype, device=dev)
    rc = load().nt_embedding(_dtype_code(W), ids.numel(), dm, vocab, _p(ids), _p(W), _p(out), _stream(dev))
    _check("nt_embedding", rc)
    return out


def lm_head(x: Tensor, gamma: Tensor, W: Tensor, workspace: Optional[Tensor] = None,
            out: Optional[Tensor] = None) -> Tensor:
    """Final RMSNorm + tied lm_head (model.py:283-284): x [..., dm] -> logits [..., vocab] in x.dtype
    (written into `out`, a contiguous tensor of that shape, when given)."""
    dev = _require_cuda(x, gamma, W)
    a = x.dtype
    dm = x.shape[-1]
    vocab = W.shape[0]
    M = x.numel() // dm
    x2, g2, W2 = _c(x), _c(gamma, a), _c(W, a)
    if out is not None:
        if out.dtype != a or not out.is_contiguous() or out.numel() != M * vocab:
            raise ValueError("out must be a contiguous [..., vocab] tensor in x.dtype")
        logits = out
    else:
        logits = torch.empty((*x.shape[:-1], vocab), dtype=a, device=dev)
    L = load()
    nbytes = L.nt_lm_head_workspace_bytes(_DT[a], M, dm, vocab)
    ws = workspace if (workspace is not None and workspace.numel() >= nbytes) else _workspace(nbytes, dev)
    rc = L.nt_lm_head(_DT[a], M, dm, vocab, _p(x2), _p(g2), _p(W2), _p(logits), _p(ws), ws.numel(), _stream(dev))
    _check("nt_lm_head", rc)
    return logits


def launch_count() -> int:
    """Kernels this library has launched in this process (nt_launch_count)."""
    return int(load().nt_launch_count())


def bounded_wait_check(limit_ns: int, device: Optional[torch.device] = None) -> None:
    """Launch the bounded-wait check on the current stream (nt_bounded_wait_check)."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    _check("nt_bounded_wait_check", load().nt_bounded_wait_check(int(limit_ns), _stream(dev)))


def device_error_flags(device: int = 0, clear: bool = True) -> int:
    """Read the device error word set by kernels whose bounded waits expired (synchronises)."""
    v = ctypes.c_uint(0)
    _check("nt_get_error_flag", load().nt_get_error_flag(device, ctypes.byref(v), 1 if clear else 0))
    return int(v.value)
