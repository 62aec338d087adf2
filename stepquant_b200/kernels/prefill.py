"""Prefill: the state pass that produces a prompt's first state (GDN and KDA).

The reference runs SGLang's chunk kernel (``TritonGDNKernel.extend``) between
``PackedStatePool.decode`` and ``PackedStatePool.encode``
(stepquant/sglang/runtime.py:193-202); the recurrence it evaluates is
core.delta_step token by token, as the reference's own
``adapters.RecurrentKernel`` (stepquant/adapters.py:36-60) applies it.  Here
``sq_gdn_prefill`` evaluates it in 64-token chunks (WY/UT form) on tensor cores
with bf16 operands and fp32 accumulation and an fp32 state.  For KDA layers
(per-key-channel decay) the reference hook calls SGLang's KDA chunk kernel the
same way; here ``sq_kda_prefill`` (``chunk_kda``) applies the recurrence token
by token with each state held in fp32 registers.

``chunk_gated_delta_rule`` and ``chunk_kda`` keep the keyword names of that recurrent kernel
(``initial_state``, ``output_final_state``, ``use_qk_l2norm_in_kernel``,
``scale``, ``cu_seqlens``); ``PackedStatePool.extend`` is the decode -> chunk
pass -> encode sequence of the reference hook.
"""
import ctypes

import torch

from .. import _native as N


def _rows(x, name):
    """[1, T, heads, dim] or [T, heads, dim] -> bf16 [T, heads, dim] with unit inner stride."""
    if x.dim() == 4:
        if x.shape[0] != 1:
            raise ValueError(f"{name}: expected a leading batch of 1 (concatenated sequences)")
        x = x[0]
    if x.dim() != 3:
        raise ValueError(f"{name}: expected [tokens, heads, dim]")
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    if x.stride(-1) != 1 or x.stride(1) != x.shape[2] or (x.stride(0) * 2) % 16 or x.data_ptr() % 16:
        x = x.contiguous()
    return x


def _gates(x, tokens, heads, name):
    if x.dim() == 3:
        if x.shape[0] != 1:
            raise ValueError(f"{name}: expected a leading batch of 1")
        x = x[0]
    if tuple(x.shape) != (tokens, heads):
        raise ValueError(f"{name}: expected [tokens, heads] = {(tokens, heads)}, got {tuple(x.shape)}")
    return x.float().contiguous()


def _channel_gates(x, tokens, heads, keys):
    if x.dim() == 4:
        if x.shape[0] != 1:
            raise ValueError("g: expected a leading batch of 1")
        x = x[0]
    if tuple(x.shape) != (tokens, heads, keys):
        raise ValueError(f"g: expected [tokens, heads, keys] = {(tokens, heads, keys)}, got {tuple(x.shape)}")
    x = x.float().contiguous()
    if x.data_ptr() % 16:
        x = x.clone()
    return x


def _prefill(kda, q, k, v, g, beta, scale, initial_state, output_final_state, use_qk_l2norm_in_kernel,
             cu_seqlens, check):
    batched = v.dim() == 4
    qr, kr, vr = _rows(q, "q"), _rows(k, "k"), _rows(v, "v")
    tokens, heads, values = vr.shape
    qk_heads, keys = qr.shape[1], qr.shape[2]
    if tuple(kr.shape) != (tokens, qk_heads, keys) or qr.shape[0] != tokens:
        raise ValueError("q, k and v must cover the same tokens, q and k the same heads")
    if heads % qk_heads:
        raise ValueError("value heads must be a multiple of qk heads")
    if keys != 128 or values != 128:
        raise NotImplementedError("the prefill passes are built for keys = values = 128")
    device = vr.device
    N.require_cuda(qr, kr, vr)
    gr = _channel_gates(g, tokens, heads, keys) if kda else _gates(g, tokens, heads, "g")
    br = _gates(beta, tokens, heads, "beta")
    if cu_seqlens is None:
        cu_seqlens = torch.tensor([0, tokens], device=device, dtype=torch.int32)
    cu = cu_seqlens.to(device=device, dtype=torch.int32).contiguous()
    seqs = cu.numel() - 1
    if seqs < 0:
        raise ValueError("cu_seqlens needs at least one entry")
    final = torch.empty(seqs, heads, keys, values, device=device, dtype=torch.float32)
    init = None
    if initial_state is not None:
        if tuple(initial_state.shape) != (seqs, heads, keys, values):
            raise ValueError(f"initial_state must be {(seqs, heads, keys, values)}")
        init = initial_state.float().contiguous()
    out = torch.empty(tokens, heads, values, device=device, dtype=torch.bfloat16)
    if kda:
        workspace = None
    else:
        workspace = torch.empty(max(N.lib().sq_gdn_prefill_workspace_bytes(tokens, seqs, heads), 1), device=device,
                                dtype=torch.uint8)
    status = torch.zeros(1, device=device, dtype=torch.int32)
    args = N.SqPrefillArgs(qr.data_ptr(), kr.data_ptr(), vr.data_ptr(), qr.stride(0), kr.stride(0), vr.stride(0),
                           N.SQ_BF16, qk_heads, heads, keys, values, 1 if use_qk_l2norm_in_kernel else 0,
                           keys ** -0.5 if scale is None else float(scale), seqs, tokens, cu.data_ptr(), gr.data_ptr(),
                           br.data_ptr(), init.data_ptr() if init is not None else None, final.data_ptr(),
                           out.data_ptr(), workspace.data_ptr() if workspace is not None else None,
                           workspace.numel() if workspace is not None else 0, status.data_ptr())
    entry = N.lib().sq_kda_prefill if kda else N.lib().sq_gdn_prefill
    N.check(entry(ctypes.byref(args), N.stream_handle()))
    if check and int(status.item()) & N.SQ_STATUS_TIMEOUT:
        raise RuntimeError("chunked prefill: a bounded device wait gave up; results are incomplete")
    if batched:
        out = out.unsqueeze(0)
    return out, (final if output_final_state else None)


def chunk_gated_delta_rule(q, k, v, g, beta, *, scale=None, initial_state=None, output_final_state=True,
                           use_qk_l2norm_in_kernel=True, cu_seqlens=None, check=True):
    """GDN prefill over concatenated sequences.

    q, k: [1, T, HK, 128] or [T, HK, 128]; v: [.., T, H, 128] (bf16; other
    dtypes are converted); g (log decay), beta: [.., T, H]; cu_seqlens: int
    [N + 1] sequence boundaries (default: one sequence of T tokens);
    initial_state: [N, H, 128, 128] fp32 or None (zeros).  Returns
    (o [.., T, H, 128] bf16 shaped like v, final_state [N, H, 128, 128] fp32
    or None when ``output_final_state`` is false).  With ``check`` the call
    waits for the device and raises RuntimeError if a bounded device wait gave
    up (SQ_STATUS_TIMEOUT); without it the call is asynchronous.
    """
    return _prefill(False, q, k, v, g, beta, scale, initial_state, output_final_state, use_qk_l2norm_in_kernel,
                    cu_seqlens, check)


def chunk_kda(q, k, v, g, beta, *, scale=None, initial_state=None, output_final_state=True,
              use_qk_l2norm_in_kernel=True, cu_seqlens=None, check=True):
    """KDA prefill over concatenated sequences: as ``chunk_gated_delta_rule``
    with g the log decay per key channel, [1, T, H, 128] or [T, H, 128].

    ``sq_kda_prefill`` keeps each (sequence, head) state in fp32 registers and
    applies core.delta_step token by token (no device waits; ``check`` only
    synchronises)."""
    return _prefill(True, q, k, v, g, beta, scale, initial_state, output_final_state, use_qk_l2norm_in_kernel,
                    cu_seqlens, check)
