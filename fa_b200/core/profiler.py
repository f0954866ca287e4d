"""In-process device-time profiling (CUDA counterpart of the reference
core/profiler.py, which drives ``torch_npu.profiler`` and parses
``kernel_details.csv``).

``profile_case_us`` keeps the reference signature and semantics: warm-ups,
then ``iters`` calls per backend inside one profiler session, and the mean
device duration of the kernels attributed to each backend.  Attribution uses
``_match_backend`` unchanged: exact symbols first (``kernel_names``), then,
for backends without an exact symbol, the directory name or ``op_type`` as a
substring of the kernel name.  The B200 kernels are named
``b200_fa_fp16_kernel`` / ``b200_fa_fp32_kernel``, so they match their
directories.  A backend whose work is spread over library kernels with
unrelated names (the FP32 torch reference) gets no kernel match; for it the
mean per-call time is taken with CUDA events instead.
"""


def _match_backend(name, backend_names, op_types, kernel_names):
    """Exact symbols first; substring/op_type fallback only for backends without one."""
    for n in backend_names:
        if name == kernel_names.get(n, f"{n}_kernel"):
            return n
    for n in backend_names:
        if n in kernel_names:
            continue
        op = op_types.get(n, "")
        if n in name or (op and op in name):
            return n
    return None


def _kernel_base_name(name):
    """'b200_fa_fp16_kernel(b200fa::FwdParams)' -> 'b200_fa_fp16_kernel'."""
    return name.split("(", 1)[0].strip()


def _event_times_us(call, iters):
    import torch

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        call()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) * 1000.0 / iters


def profile_case_us(calls, backend_names, iters=20, warmup=3, op_types=None, kernel_names=None):
    """Mean device microseconds per backend: {name: avg_us or None}."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    op_types = op_types or {}
    kernel_names = kernel_names or {}
    active = [n for n in backend_names if n in calls]
    for n in active:
        for _ in range(warmup):
            calls[n]()
    torch.cuda.synchronize()

    durations = {}
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for n in active:
            for _ in range(iters):
                calls[n]()
            torch.cuda.synchronize()
    for evt in prof.events():
        if evt.device_type != torch.autograd.DeviceType.CUDA:
            continue
        name = _kernel_base_name(evt.name)
        n = _match_backend(name, backend_names, op_types, kernel_names)
        us = evt.time_range.elapsed_us()
        if n is not None and n in calls and us > 0:
            durations.setdefault(n, []).append(us)

    result = {}
    for n in backend_names:
        ds = durations.get(n)
        if ds:
            result[n] = sum(ds) / len(ds)
        elif n in calls:
            result[n] = _event_times_us(calls[n], iters)
        else:
            result[n] = None
    return result
