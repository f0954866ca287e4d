"""CPU/FP32 oracle for the attention forward -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline
leg (and its ``--impl reference`` arm) may import this module, and only as
the checker or as the timed CPU baseline.  The product path (``fa_b200``)
never imports it.

What it restates
----------------
* ``attention_fp32`` -- the reference's FP32 formula ``ref_flash_attn``
  (backends/expert_v2/impl_tl.py:701-717): upcast Q/K/V to FP32, expand the
  KV heads with ``repeat_interleave(Hq/Hkv, dim=1)`` (the GQA map
  kv = h / (Hq/Hkv) of panel_kernel.h:274), non-causal softmax(Q K^T * scale)
  V with scale = D**-0.5 (problem/cases.py:26-27).  Computed block-wise over
  query rows and heads so memory stays bounded; returns FP32 (the reference
  casts to FP16 at the end -- ``to_fp16`` does that step).  TF32 is disabled
  when it runs on a CUDA device.
* ``attention_f64`` -- the same formula in float64 NumPy, for small cases:
  the most exact statement of the operator, used to pin the FP32 one.
* ``attention_rows_fp32`` -- selected query rows only, for spot checks of
  full-size problems.
* ``online_state_f64`` -- the per-block online-softmax state (m, l, alpha,
  z, O) that the kernel's debug capture records, in float64.
* ``attention_sdpa_fp32`` -- the reference formula in its own form
  (repeat_interleave + FP32 ``scaled_dot_product_attention``): the CPU path
  that bench.py times as the CPU baseline.

Pinning
-------
tests/golden/ holds vectors produced by running the reference's own
``ref_flash_attn`` (extracted from its source file) on seeded inputs in the
build container (script: tests/golden/make_golden.py).  tests/test_oracle.py
checks both restatements against every vector.  The closed NPU operator
(``torch_npu.npu_fusion_attention``, backends/npu_fa/backend.py:36-49) cannot
run here; parity with it is established only through the reference's FP32
formula, which the reference documents as agreeing with it within 1e-4
(backends/npu_fa/backend.py:4-7).
"""

from __future__ import annotations

import numpy as np
import torch


def _expand_kv(k: torch.Tensor, v: torch.Tensor, heads_q: int):
    if k.shape[1] != heads_q:
        rep = heads_q // k.shape[1]
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
    return k, v


@torch.no_grad()
def attention_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None,
                   rows_per_block: int = 1024, causal: bool = False) -> torch.Tensor:
    """FP32 O[B,Hq,Nq,D] = softmax(Q K^T * scale) V, on q's device.

    ``causal``: query row i attends keys 0..i (top-left aligned mask, the
    convention of torch's ``is_causal``) -- the B200 build's optional causal
    mode; the reference operator itself is non-causal."""
    B, Hq, Nq, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    scale = D ** -0.5 if scale is None else scale
    prev_tf32 = None
    if q.is_cuda:
        prev_tf32 = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
    try:
        out = torch.empty((B, Hq, Nq, D), dtype=torch.float32, device=q.device)
        for b in range(B):
            for h in range(Hq):
                kf = k[b, h // G].float()
                vf = v[b, h // G].float()
                for r0 in range(0, Nq, rows_per_block):
                    qf = q[b, h, r0:r0 + rows_per_block].float()
                    s = (qf @ kf.T) * scale
                    if causal:
                        rows = torch.arange(r0, r0 + qf.shape[0], device=s.device)[:, None]
                        cols = torch.arange(kf.shape[0], device=s.device)[None, :]
                        s = s.masked_fill(cols > rows, float("-inf"))
                    s -= s.amax(dim=-1, keepdim=True)
                    p = torch.exp(s)
                    out[b, h, r0:r0 + rows_per_block] = (p @ vf) / p.sum(dim=-1, keepdim=True)
        return out
    finally:
        if prev_tf32 is not None:
            torch.backends.cuda.matmul.allow_tf32 = prev_tf32


@torch.no_grad()
def attention_rows_fp32(q, k, v, rows, scale: float | None = None) -> torch.Tensor:
    """FP32 output of selected (b, h, row) query rows: rows is an int tensor [n, 3]."""
    D = q.shape[-1]
    G = q.shape[1] // k.shape[1]
    scale = D ** -0.5 if scale is None else scale
    out = torch.empty((rows.shape[0], D), dtype=torch.float32, device=q.device)
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for i, (b, h, r) in enumerate(rows.tolist()):
            kf = k[b, h // G].float()
            s = (q[b, h, r].float() @ kf.T) * scale
            p = torch.softmax(s, dim=-1)
            out[i] = p @ v[b, h // G].float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32
    return out


def attention_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float | None = None) -> np.ndarray:
    """float64 NumPy restatement (small cases)."""
    B, Hq, Nq, D = q.shape
    G = Hq // k.shape[1]
    scale = D ** -0.5 if scale is None else scale
    out = np.empty((B, Hq, Nq, D), dtype=np.float64)
    for b in range(B):
        for h in range(Hq):
            qf = q[b, h].astype(np.float64)
            kf = k[b, h // G].astype(np.float64)
            vf = v[b, h // G].astype(np.float64)
            s = qf @ kf.T * scale
            s -= s.max(axis=-1, keepdims=True)
            p = np.exp(s)
            out[b, h] = (p @ vf) / p.sum(axis=-1, keepdims=True)
    return out


def online_state_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float | None = None,
                     block: int = 128, threshold: float = 8.0) -> dict:
    """float64 restatement of the per-block online-softmax state that the
    debug capture records, for small cases.

    The recurrence is the reference's (CCE ``Stats``,
    op_kernel/vector_output.h:94-106 of the cce_fa_nqkq_nz_resident backend:
    l = z at the first packet, l = alpha*l + z after it; O likewise), here
    over key blocks of ``block`` keys with the lazy reference maximum of the
    B200 kernel: in the log2 domain (scores times scale*log2(e)) the maximum
    m moves to a block's maximum only when that exceeds m by more than
    ``threshold``; then alpha = 2^(m_old - m_new) (0 at the first block),
    else alpha = 1.  Per block: z = sum 2^(s - m) over the block's keys,
    l = alpha*l + z, O = alpha*O + fp16(2^(s - m)) V (P is rounded to FP16
    before the P V product, as the kernel does).

    Returns {m, l, alpha, z: [B, Hq, n_blocks, Nq]; o: [..., D];
    margin: [B, Hq, Nq]} where margin is the smallest distance of a
    block maximum from the move threshold (a decision closer than the
    arithmetic's error may go either way).
    """
    B, Hq, Nq, D = q.shape
    Nk = k.shape[2]
    G = Hq // k.shape[1]
    scale = D ** -0.5 if scale is None else scale
    nb = -(-Nk // block)
    log2e = 1.0 / np.log(2.0)
    out = {name: np.empty((B, Hq, nb, Nq)) for name in ("m", "l", "alpha", "z")}
    out["o"] = np.empty((B, Hq, nb, Nq, D))
    out["margin"] = np.full((B, Hq, Nq), np.inf)
    for b in range(B):
        for h in range(Hq):
            s = (q[b, h].astype(np.float64) @ k[b, h // G].astype(np.float64).T) * (scale * log2e)
            vf = v[b, h // G].astype(np.float64)
            m = np.full(Nq, -np.inf)
            l = np.zeros(Nq)
            o = np.zeros((Nq, D))
            for j in range(nb):
                sb = s[:, j * block:(j + 1) * block]
                m_blk = sb.max(axis=1)
                gap = m_blk - (m + threshold)
                out["margin"][b, h] = np.minimum(out["margin"][b, h], np.abs(gap))
                move = gap > 0
                alpha = np.where(move, np.exp2(np.where(move, m - m_blk, 0.0)), 1.0)
                m = np.where(move, m_blk, m)
                p = np.exp2(sb - m[:, None])
                z = p.sum(axis=1)
                l = alpha * l + z
                o = alpha[:, None] * o + p.astype(np.float16).astype(np.float64) @ vf[j * block:(j + 1) * block]
                out["m"][b, h, j], out["l"][b, h, j], out["z"][b, h, j] = m, l, z
                out["alpha"][b, h, j] = 0.0 if j == 0 else alpha
                out["o"][b, h, j] = o
    return out


def to_fp16(o: torch.Tensor) -> torch.Tensor:
    """The reference's final cast (impl_tl.py:717)."""
    return o.to(torch.float16)


def errors(out: torch.Tensor, ref: torch.Tensor) -> tuple[float, float]:
    """(max-abs, mean-abs) of out - ref in FP32."""
    d = (out.float() - ref.float()).abs()
    return float(d.max()), float(d.mean())


def flops(B: int, Hq: int, Nq: int, Nk: int, D: int = 128) -> int:
    return 4 * B * Hq * Nq * Nk * D


def attention_sdpa_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """The reference formula verbatim in structure (impl_tl.py:701-717): GQA by
    repeat_interleave, FP32 scaled_dot_product_attention, default scale,
    non-causal; FP32 result (before the reference's FP16 cast).  This is the
    reference's CPU path that the CPU baseline times."""
    if k.shape[1] != q.shape[1]:
        rep = q.shape[1] // k.shape[1]
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
    return torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.float(), v.float(), attn_mask=None, dropout_p=0.0, is_causal=False)


def cpu_time_sample(B: int, Hq: int, Hkv: int, N: int, rows: int, seed: int = 0,
                    threads: int | None = None, min_seconds: float = 0.0):
    """Time the reference's CPU path (``attention_sdpa_fp32``) on the host cores
    over a bounded sample of a case.

    The sample is ``rows`` query rows of one (b, h) against the full Nk keys;
    the work is linear in Nq, so throughput carries over to the whole case.
    Repeats until ``min_seconds`` elapsed.  Returns (tflops, seconds, reps,
    threads, sample description).
    """
    import time

    if threads:
        torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((1, 1, rows, 128), generator=g).half()
    k = torch.randn((1, 1, N, 128), generator=g).half()
    v = torch.randn((1, 1, N, 128), generator=g).half()
    attention_sdpa_fp32(q, k, v)  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        attention_sdpa_fp32(q, k, v)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    fl = flops(1, 1, rows, N) * reps
    desc = (f"{rows} query rows x 1 head x Nk={N} keys of B={B},Hq={Hq},Hkv={Hkv},N={N} "
            f"(FP32 scaled_dot_product_attention, {reps} reps), throughput scaled linearly in Nq")
    return fl / el / 1e12, el, reps, torch.get_num_threads(), desc


__all__ = ["attention_fp32", "attention_sdpa_fp32", "attention_rows_fp32", "attention_f64", "to_fp16",
           "errors", "flops", "cpu_time_sample"]

