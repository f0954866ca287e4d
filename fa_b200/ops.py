"""Torch-facing attention operator over ``libb200fa.so``.

``Operator`` is the B200 counterpart of the reference CCE binding's
``Operator`` (backends/cce_fa_nqkq_nz_resident_v13_q768_pool_i4_p128/
binding.py:139-242): same call signature ``op(q, k, v) -> O``, same argument
checks and ``ValueError`` messages (binding.py:219-231), workspace owned and
reused by the operator (binding.py:166-187, 208-209).  Differences, all
relaxations: any Nq >= 1 and Nk >= 1 is accepted (the reference requires
Nq % 128 == 0 and Nk % 512 == 0), and a unit range selects a shard of the
(b, hq, 128-row query block) grid for multi-GPU runs.

PyTorch is used for device memory and streams only; all arithmetic runs in
the sm_100a kernels.  There is no CPU or eager fallback: a missing library or
a non-CUDA tensor raises.
"""

from __future__ import annotations

import math

import torch

from . import lib
from .shard import pieces, row_range

HEAD_DIM = 128
BLOCK_M = 128


def _geometry(q, k, v):
    """Validate like binding.py:219-231 and return (B, Hq, Hkv, Nq, Nk)."""
    if q.ndim != 4 or k.ndim != 4 or v.shape != k.shape:
        raise ValueError("Q/K/V must be [B,H,N,128]")
    b, h, nq, d = q.shape
    if (min(q.shape) <= 0 or min(k.shape) <= 0 or k.shape[0] != b or d != HEAD_DIM
            or k.shape[3] != HEAD_DIM or h % k.shape[1]):
        raise ValueError("invalid attention geometry")
    nk = k.shape[2]
    if max(nq, nk) > 2**31 - 1:
        raise ValueError("unsupported query/key tail")
    for t in (q, k, v):
        if (t.device.type != "cuda" or t.device != q.device or t.dtype != torch.float16
                or not t.is_contiguous()):
            raise ValueError("Q/K/V must be contiguous FP16 on the same CUDA device")
    return b, h, k.shape[1], nq, nk


class Operator:
    """``op(q, k, v) -> O``: non-causal GQA attention forward, FP16 in/out.

    variant: "fp16" (row sums over the FP16 P in FP16 partial sums, after the
             CCE FP16 kernel) or "fp32" (FP32 softmax, the CCE FP32 kernel).
    debug:   run the checking build (libb200fa_debug.so): same results, plus
             bounds, index and layout checks before every copy and a check of
             the roles' key-block counts at exit, reported as
             B200FA_DEV_BOUNDS / B200FA_DEV_PHASE in ``status``.
    """

    def __init__(self, variant: str = "fp16", *, timeout_us: int = 0, trace: bool = False,
                 max_ctas: int = 0, debug: bool = False):
        if variant not in lib.VARIANTS:
            raise ValueError(f"variant must be one of {sorted(lib.VARIANTS)}")
        self.variant = variant
        self.variant_id = lib.VARIANTS[variant]
        self.timeout_us = int(timeout_us)
        self.flags = lib.FLAG_TRACE if trace else 0
        self.max_ctas = int(max_ctas)
        self.debug = bool(debug)
        self.workspaces = {}  # device -> uint8 tensor (zeroed once)
        self._streams = {}    # device -> (upload, download) streams of forward_host
        lib.load(debug=self.debug)

    @property
    def kernel_name(self) -> str:
        return lib.kernel_name(self.variant_id)

    def workspace(self, device) -> torch.Tensor:
        ws = self.workspaces.get(device)
        if ws is None:
            ws = torch.zeros(lib.WS_BYTES, dtype=torch.uint8, device=device)
            self.workspaces[device] = ws
        return ws

    def __call__(self, q, k, v, *, scale: float | None = None, out: torch.Tensor | None = None,
                 unit_range: tuple[int, int] | None = None, flags: int = 0,
                 capture: torch.Tensor | None = None, causal: bool = False) -> torch.Tensor:
        """O = softmax(Q K^T * scale) V.  ``causal``: query row i attends keys
        0..i only (top-left aligned, as torch's ``is_causal``; an addition,
        the reference's operator is non-causal).  ``capture`` (FP32, at least
        ``capture_bytes(...)`` bytes, on Q's device) turns on the debug
        capture of the per-block online-softmax state (``capture_view``)."""
        if causal:
            flags |= lib.FLAG_CAUSAL
        B, Hq, Hkv, Nq, Nk = _geometry(q, k, v)
        if out is None:
            out = torch.empty_like(q)
        elif out.shape != q.shape or out.dtype != torch.float16 or not out.is_contiguous() \
                or out.device != q.device:
            raise ValueError("out must be a contiguous FP16 tensor shaped like Q on Q's device")
        units = lib.num_units(B, Hq, Nq)
        begin, end = (0, units) if unit_range is None else (int(unit_range[0]), int(unit_range[1]))
        scale = float(HEAD_DIM ** -0.5 if scale is None else scale)
        ws = self.workspace(q.device)
        cap_ptr, cap_bytes, cap_flag = None, 0, 0
        if capture is not None:
            if capture.dtype != torch.float32 or not capture.is_contiguous() or capture.device != q.device:
                raise ValueError("capture must be a contiguous FP32 tensor on Q's device")
            cap_ptr, cap_bytes, cap_flag = capture.data_ptr(), capture.numel() * 4, lib.FLAG_CAPTURE
        with torch.cuda.device(q.device):
            stream = torch.cuda.current_stream(q.device).cuda_stream
            lib.fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                    B, Hq, Hkv, Nq, Nk, HEAD_DIM, scale, self.variant_id, begin, end,
                    ws.data_ptr(), ws.numel(), stream,
                    flags=self.flags | flags | cap_flag, timeout_us=self.timeout_us, max_ctas=self.max_ctas,
                    capture_ptr=cap_ptr, capture_bytes=cap_bytes, debug=self.debug)
        return out

    def forward_host(self, q_host, k_host, v_host, out_host, *, q_dev, k_dev, v_dev, o_dev,
                     scale: float | None = None, unit_range: tuple[int, int] | None = None,
                     chunks: int = 3, causal: bool = False) -> tuple[int, int]:
        """O = attention(Q, K, V) from pinned host buffers into a pinned host
        buffer, with the copies overlapped with the kernel.

        The unit range is cut into ``chunks`` contiguous pieces (whole work
        items of two query blocks, the end pieces quarter-sized).  On an
        upload stream, each piece's K/V heads not yet on the device go up,
        then its Q rows; the piece's kernel runs on the current stream once
        they are there, and its O rows come down on a download stream while
        the next pieces run.  Only the K/V heads the range uses are moved
        (a range inside one batch needs only that batch's heads).
        ``*_dev`` are device buffers of the full shapes; ``q_host`` and
        ``out_host`` hold either the full Q/O or only the unit range's rows
        (flattened to [rows, 128]).  Work is enqueued on the current stream,
        which also waits for the last download: synchronize it to read
        ``out_host``.  Returns the (host-to-device, device-to-host) bytes.
        """
        B, Hq, Hkv, Nq, Nk = _geometry(q_dev, k_dev, v_dev)
        units = num_units(B, Hq, Nq)
        ub, ue = (0, units) if unit_range is None else unit_range
        if not 0 <= ub <= ue <= units:
            raise ValueError(f"unit range [{ub}, {ue}) outside [0, {units})")
        R0, R1 = row_range(ub, ue, Nq)
        for name, t, ref in (("q_host", q_host, q_dev), ("k_host", k_host, k_dev), ("v_host", v_host, v_dev),
                             ("out_host", out_host, o_dev)):
            rows_only = name in ("q_host", "out_host") and tuple(t.shape) == (R1 - R0, HEAD_DIM)
            if (t.device.type != "cpu" or not t.is_pinned() or t.dtype != ref.dtype
                    or not (t.shape == ref.shape or rows_only)):
                raise ValueError(f"{name} must be a pinned host tensor shaped like its device buffer")
        dev = q_dev.device
        cur = torch.cuda.current_stream(dev)
        s_in, s_out = self._copy_streams(dev)
        qd, od = q_dev.view(-1, HEAD_DIM), o_dev.view(-1, HEAD_DIM)
        qh, oh = q_host.view(-1, HEAD_DIM), out_host.view(-1, HEAD_DIM)
        kd, vd = k_dev.view(B * Hkv, Nk, HEAD_DIM), v_dev.view(B * Hkv, Nk, HEAD_DIM)
        kh, vh = k_host.view(B * Hkv, Nk, HEAD_DIM), v_host.view(B * Hkv, Nk, HEAD_DIM)
        qo = 0 if q_host.numel() == q_dev.numel() else R0  # host row of flattened row r: r - qo
        oo = 0 if out_host.numel() == o_dev.numel() else R0
        nqb, group = -(-Nq // BLOCK_M), Hq // Hkv

        def kv_head(u):  # K/V head (b*Hkv + kvh) of unit u
            bh = u // nqb
            return (bh // Hq) * Hkv + (bh % Hq) // group

        bounds = pieces(ub, ue, chunks)
        n = len(bounds) - 1
        h2d = d2h = 0
        kv_done = None  # K/V heads [first, kv_done) of the range are uploaded
        s_in.wait_stream(cur)  # the device buffers are free once earlier work on `cur` is
        ev_q = []
        with torch.cuda.stream(s_in):
            for c in range(n):
                a, b = bounds[c], bounds[c + 1]
                if b > a:
                    first, last = kv_head(a), kv_head(b - 1) + 1
                    lo = first if kv_done is None else max(first, kv_done)
                    if last > lo:
                        kd[lo:last].copy_(kh[lo:last], non_blocking=True)
                        vd[lo:last].copy_(vh[lo:last], non_blocking=True)
                        h2d += 2 * (last - lo) * Nk * HEAD_DIM * 2
                        kv_done = last
                r0, r1 = row_range(a, b, Nq)
                qd[r0:r1].copy_(qh[r0 - qo:r1 - qo], non_blocking=True)
                h2d += (r1 - r0) * HEAD_DIM * 2
                ev_q.append(s_in.record_event())
        for c in range(n):
            cur.wait_event(ev_q[c])
            self(q_dev, k_dev, v_dev, scale=scale, out=o_dev, unit_range=(bounds[c], bounds[c + 1]), causal=causal)
            s_out.wait_stream(cur)
            r0, r1 = row_range(bounds[c], bounds[c + 1], Nq)
            with torch.cuda.stream(s_out):
                oh[r0 - oo:r1 - oo].copy_(od[r0:r1], non_blocking=True)
            d2h += (r1 - r0) * HEAD_DIM * 2
        cur.wait_stream(s_out)
        return h2d, d2h

    def _copy_streams(self, dev):
        key = ("copy_streams", dev.index)
        streams = self._streams.get(key)
        if streams is None:
            streams = self._streams[key] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
        return streams

    CAPTURE_LIMIT = 256 << 20  # bytes; the reference restricts its capture the same way

    @staticmethod
    def capture_buffer(q, k) -> torch.Tensor:
        """A NaN-filled capture buffer for Q/K's shapes (entries outside the
        unit range stay NaN).  Debug capture is for small inputs only."""
        B, Hq, Nq, _ = q.shape
        nbytes = lib.capture_bytes(B, Hq, Nq, k.shape[2])
        if nbytes > Operator.CAPTURE_LIMIT:
            raise ValueError("debug capture is restricted to small inputs (at most 256 MiB)")
        return torch.full((nbytes // 4,), float("nan"), dtype=torch.float32, device=q.device)

    @staticmethod
    def capture_view(capture: torch.Tensor, q, k) -> dict:
        """The capture buffer as {m, l, alpha, z: [B, Hq, n_blocks, Nq];
        o, o_partial: [B, Hq, n_blocks, Nq, D]}.  ``o`` is the running
        (unnormalised) output after each key block; ``o_partial`` the block's
        own P V product, O_j - alpha_j O_(j-1), derived here."""
        B, Hq, Nq, D = q.shape
        nb = -(-k.shape[2] // lib.BLOCK_KEYS)
        rows = B * Hq * nb * Nq
        planes = capture[:4 * rows].view(4, B, Hq, nb, Nq)
        o = capture[4 * rows:4 * rows + rows * D].view(B, Hq, nb, Nq, D)
        prev = torch.cat([torch.zeros_like(o[:, :, :1]), o[:, :, :-1]], dim=2)
        o_partial = o - planes[2].unsqueeze(-1) * prev
        return {"m": planes[0], "l": planes[1], "alpha": planes[2], "z": planes[3],
                "o": o, "o_partial": o_partial}

    def status(self, device) -> tuple[int, int, int, int]:
        """Synchronize and read the device status header {status, site, cta, 0}."""
        ws = self.workspace(torch.device(device))
        with torch.cuda.device(ws.device):
            return lib.read_status(ws.data_ptr(), torch.cuda.current_stream(ws.device).cuda_stream)

    def reset_status(self, device) -> None:
        ws = self.workspace(torch.device(device))
        with torch.cuda.device(ws.device):
            lib.reset_status(ws.data_ptr(), torch.cuda.current_stream(ws.device).cuda_stream)

    def timeline(self, device):
        """The first pair's clock64 stamps of the last B200FA_FLAG_TIMELINE call
        as an int64 tensor [2 ranks, TIMELINE_ROLES, TIMELINE_BLOCKS, 8 events]
        (synchronizes)."""
        ws = self.workspace(torch.device(device))
        torch.cuda.synchronize(ws.device)
        raw = ws[lib.WS_TIMELINE_OFFSET:lib.WS_TIMELINE_OFFSET + lib.WS_TIMELINE_BYTES]
        return raw.view(torch.int64).view(2, lib.TIMELINE_ROLES, lib.TIMELINE_BLOCKS, 8).cpu()

    def trace(self, device) -> list[dict]:
        """Per-CTA trace records of the last traced call (synchronizes).

        Both CTAs of a pair report the pair's item count; ``rank`` is the
        CTA's rank in its pair."""
        ws = self.workspace(torch.device(device))
        torch.cuda.synchronize(ws.device)
        raw = ws[lib.WS_HEADER_BYTES:lib.WS_TIMELINE_OFFSET].view(torch.int32).view(-1, 8).cpu()
        recs = []
        for r in raw.tolist():
            t0 = (r[2] & 0xFFFFFFFF) | ((r[3] & 0xFFFFFFFF) << 32)
            t1 = (r[4] & 0xFFFFFFFF) | ((r[5] & 0xFFFFFFFF) << 32)
            if t1 == 0:
                continue
            recs.append({"smid": r[0], "items": r[1], "t_start_ns": t0, "t_end_ns": t1, "rank": r[6]})
        return recs


_OPS = {}


def attention(q, k, v, *, variant: str = "fp16", scale: float | None = None, out=None,
              unit_range=None) -> torch.Tensor:
    """Functional form: O = softmax(Q K^T * scale) V with GQA (Hq % Hkv == 0)."""
    op = _OPS.get(variant)
    if op is None:
        op = _OPS[variant] = Operator(variant)
    return op(q, k, v, scale=scale, out=out, unit_range=unit_range)


def flops(B: int, Hq: int, Nq: int, Nk: int, D: int = HEAD_DIM) -> int:
    """QK^T and PV FLOPs, 4*B*Hq*Nq*Nk*D (reference README.md:86)."""
    return 4 * B * Hq * Nq * Nk * D


def num_units(B: int, Hq: int, Nq: int) -> int:
    return B * Hq * math.ceil(Nq / BLOCK_M)

