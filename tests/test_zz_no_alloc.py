"""xq4_linear_sharded_noalloc: the sharded linear for callers that cannot
allocate device memory when they run the op (a serving engine that reserved
the GPU's memory up front, a decode loop that cannot afford the device-wide
synchronisation of cudaFree, a foreign-language caller with no device
allocator).  It stages the m > 1 gather through a fixed scratch array inside
the library instead of a caller workspace.

Checked on one GPU with a one-rank communicator, through the C ABI, against
xq4_linear_sharded (with a workspace) on the same inputs, for two calls in a
row (the scratch keeps the previous call's contents), within the parity bar of
the other tests; plus the rejection of sizes beyond the scratch.  This file is
collected last so that a run stopping at the first failure has already run
every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from xnpu_b200 import _lib, hal, lib, synth
from xnpu_b200._lib import check
from test_gpu_kernels import import_planes, rel_metrics

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def one_rank(dev):
    """A communicator of one rank on the test device, warmed up with one
    collective (the workspace entry point) before the no-allocation calls."""
    L = lib()
    uid = (ctypes.c_char * _lib.XQ4_UNIQUE_ID_BYTES)()
    check(L.xq4_comm_unique_id(ctypes.addressof(uid)))
    comm = ctypes.c_void_p()
    check(L.xq4_comm_init(dev.handle, 0, 1, ctypes.addressof(uid), ctypes.byref(comm)))
    yield comm
    check(L.xq4_comm_destroy(comm))


@pytest.mark.parametrize("m,f32", [(1, 0), (3, 0), (3, 1), (20, 0)])
def test_noalloc_matches_workspace_entry_point(dev, one_rank, m, f32):
    L = lib()
    n, k = 4096, 4096
    q = synth.unpack_codes_signed(synth.synth_codes(n, k, 880))
    s = synth.synth_scales(n, k, 880)
    w = import_planes(dev, q, s)
    dt = torch.float32 if f32 else torch.bfloat16
    st = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # two calls in a row, different activations
        x = synth.synth_x(m, k, 881 + 10 * m + call)
        xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)
        ref = torch.empty((m, n), dtype=dt, device="cuda")
        ws = torch.empty((m, n), dtype=dt, device="cuda")
        check(L.xq4_linear_sharded(one_rank, w.handle, xd.data_ptr(), ref.data_ptr(), ws.data_ptr(), m, f32, st))
        got = torch.full((m, n), float("nan"), dtype=dt, device="cuda")
        check(L.xq4_linear_sharded_noalloc(one_rank, w.handle, xd.data_ptr(), got.data_ptr(), m, f32, st))
        torch.cuda.synchronize()
        a, b = got.float().cpu().numpy(), ref.float().cpu().numpy()
        assert np.isfinite(a).all(), f"call {call}: output not fully written"
        max_rel, mae, _ = rel_metrics(a, b)
        assert max_rel <= 1e-2 and mae <= 1e-3, (call, max_rel, mae)
    w.destroy()


def test_noalloc_rejects_sizes_beyond_the_scratch(dev, one_rank):
    L = lib()
    n, k = 4096, 4096
    q = synth.unpack_codes_signed(synth.synth_codes(n, k, 890))
    s = synth.synth_scales(n, k, 890)
    w = import_planes(dev, q, s)
    m = _lib.XQ4_NOALLOC_SCRATCH_BYTES // (n * 2) + 1  # one token row too many for bf16 output
    x = torch.zeros((m, k), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
    rc = L.xq4_linear_sharded_noalloc(one_rank, w.handle, x.data_ptr(), y.data_ptr(), m, 0,
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.XQ4_EINVAL
    assert b"scratch" in L.xq4_last_error_string()
    w.destroy()
