"""The allocation-free calibration entry point matches the workspace entry point.

``kvc_calibration_accumulate_noalloc`` serves callers that cannot hand the
library device memory (a process whose GPU memory is already reserved, or a
host that binds only the C ABI).  Called through the C ABI twice in a row, its
running fp64 sums must equal those of ``kvc_calibration_accumulate`` given a
caller-owned workspace, also for token counts whose full-parallelism workspace
is far larger than the fixed scratch (the launch then plans fewer partial rows);
a head geometry whose single partial row exceeds the scratch must be refused
before anything is launched.  This file is collected last on purpose.
"""

from __future__ import annotations

import pytest
import torch

from vllm_ascend_kvcompress import _native as N

pytestmark = pytest.mark.gpu


def _sums(heads: int, f: int, p: int):
    z = lambda w: torch.zeros(heads, w, dtype=torch.float64, device="cuda")
    return z(f), z(f), z(f), (z(p) if p else None)


def _ptr(t):
    return None if t is None else t.data_ptr()


@pytest.mark.parametrize("heads,head_dim,rot,sizes", [
    (40, 128, 128, (6000, 777)),
    (16, 256, 64, (6000, 777)),
    (40, 128, 128, (80000, 131072)),  # beyond what one scratch-sized wave of 512-token partials covers
])
def test_noalloc_matches_workspace_entry_on_two_calls(heads, head_dim, rot, sizes):
    lib = N.lib()
    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream().cuda_stream
    f, p = rot // 2, head_dim - rot
    g = torch.Generator(device="cuda").manual_seed(1234)
    calls = [(torch.randn(n, heads * head_dim, generator=g, device="cuda") + 0.25).to(torch.bfloat16)
             for n in sizes]
    ref = _sums(heads, f, p)
    got = _sums(heads, f, p)
    for q in calls:
        need = lib.kvc_calibration_workspace_doubles(q.shape[0], heads, head_dim, rot)
        ws = torch.empty(need, dtype=torch.float64, device="cuda")
        rc = lib.kvc_calibration_accumulate(q.data_ptr(), N.BF16, q.shape[0], q.stride(0), heads, head_dim, rot,
                                            *(_ptr(t) for t in ref), ws.data_ptr(), ws.numel(), stream)
        assert rc == 0
        rc = lib.kvc_calibration_accumulate_noalloc(q.data_ptr(), N.BF16, q.shape[0], q.stride(0), heads, head_dim,
                                                    rot, *(_ptr(t) for t in got), stream)
        assert rc == 0
    torch.cuda.synchronize()
    for a, b in zip(got, ref):
        if b is not None:
            torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-4)


def test_noalloc_refuses_geometry_beyond_its_scratch():
    lib = N.lib()
    # one partial row holds 3 * heads * (rot/2 + head_dim - rot) doubles
    heads, head_dim, rot = 8192, 128, 128
    assert 3 * heads * (rot // 2) > N.CALIB_STATIC_SCRATCH_DOUBLES
    sums = _sums(heads, rot // 2, 0)
    q = torch.zeros(1, 8, dtype=torch.bfloat16, device="cuda")  # never read: refused up front
    rc = lib.kvc_calibration_accumulate_noalloc(q.data_ptr(), N.BF16, 1, heads * head_dim, heads, head_dim,
                                                rot, *(_ptr(t) for t in sums), torch.cuda.current_stream().cuda_stream)
    assert rc == -28
    assert b"static scratch" in lib.kvc_status_string(rc)
    # a token count far beyond one scratch-sized wave is served
    assert lib.kvc_calibration_workspace_doubles(1 << 20, 40, 128, 128) > N.CALIB_STATIC_SCRATCH_DOUBLES
