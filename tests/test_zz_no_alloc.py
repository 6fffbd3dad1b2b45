"""vx_ulysses_attn_fwd_static: the Ulysses layer with its built-in workspace.

Some hosts may not allocate device memory inside the call -- an XLA custom
call, whose device memory belongs to XLA's allocator -- so this entry point
takes no workspace and allocates nothing; it uses a fixed 32 MiB device
array instead. These tests call it through the C ABI on a one-rank
communicator and compare it with vx_ulysses_attn_fwd given a caller-owned
workspace, on two different calls in a row (the second must not depend on
what the first left in the shared array), and check that a call needing
more than 32 MiB is refused. Tolerance: max-abs 2e-2, mean-abs 2e-3 (the
outputs are expected to be identical: same kernels, same inputs).

This file is named to be collected last."""
import ctypes

import numpy as np
import pytest
import torch

from oracle.attention_ref import compare, seeded_qkv

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda().bfloat16()


def _call(entry, q, k, v, comm, valid_len=0, workspace=None):
    from vidax_b200 import _lib
    from vidax_b200.ulysses_capi import UlyssesArgs
    out = torch.empty_like(q)
    a = UlyssesArgs()
    a.q, a.k, a.v, a.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    for f, t in (("q_stride", q), ("k_stride", k), ("v_stride", v), ("o_stride", out)):
        getattr(a, f)[:] = t.stride()[:3]
    a.batch, a.seq_local, a.heads, a.head_dim = q.shape
    a.scale = float(q.shape[-1] ** -0.5)
    a.valid_len = valid_len
    if workspace is not None:
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel()
    fn = getattr(_lib.load(), entry)
    fn.argtypes = [ctypes.POINTER(UlyssesArgs), ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    rc = fn(ctypes.byref(a), comm.handle,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, out


@pytest.mark.gpu
def test_static_workspace_matches_caller_workspace_two_calls():
    from vidax_b200 import _lib
    from vidax_b200.ulysses_capi import Comm, unique_id, workspace_bytes
    comm = Comm.init(0, 1, unique_id())
    try:
        # (B, S, H, D), valid_len: the second call is smaller and masked, so
        # it would read stale bytes of the first if the layer relied on any
        for shape, valid, seed in (((2, 512, 10, 128), 0, 1501), ((1, 777, 5, 64), 700, 1502)):
            q, k, v = (_dev(x) for x in seeded_qkv(shape, seed))
            ws = torch.empty(workspace_bytes(q, 1), dtype=torch.uint8, device=q.device)
            rc, ref = _call("vx_ulysses_attn_fwd", q, k, v, comm, valid, ws)
            _lib.check(rc)
            rc, out = _call("vx_ulysses_attn_fwd_static", q, k, v, comm, valid)
            _lib.check(rc)
            torch.cuda.synchronize()
            assert _lib.device_status(clear=True) == 0
            mx, mean = compare(out.float().cpu().numpy(), ref.float().cpu().numpy())
            assert mx <= MAX_ABS and mean <= MEAN_ABS, (shape, mx, mean)
    finally:
        comm.close()


@pytest.mark.gpu
def test_static_workspace_refuses_calls_beyond_32_mib():
    from vidax_b200 import _lib
    from vidax_b200.ulysses_capi import Comm, unique_id
    comm = Comm.init(0, 1, unique_id())
    try:
        # 8 slabs of 4096 x 40 x 128 bf16 = 336 MB of workspace
        q = torch.empty((1, 4096, 40, 128), dtype=torch.bfloat16, device="cuda")
        rc, _ = _call("vx_ulysses_attn_fwd_static", q, q, q, comm)
        assert rc == _lib.VX_EINVAL
        assert "32 MiB" in _lib.load().vx_last_error().decode()
    finally:
        comm.close()
