"""xq4_linear_sharded_noalloc: the sharded linear for callers that cannot
allocate device memory when they run the op (a serving engine that reserved
the GPU's memory up front, a decode loop that cannot afford the device-wide
synchronisation of cudaFree, a foreign-language caller with no device
allocator).  It stages the m > 1 gather through a fixed scratch array inside
the library instead of a caller workspace.

Checked on one GPU with a one-rank communicator, through the C ABI, against
xq4_linear_sharded (with a workspace) on the same inputs: the same kernels
run on the same data, so the outputs must be bit-identical, for two calls in a
row (the scratch keeps the previous call's contents), on the decode GEMV
(m < 25) and on the tensor-core GEMM (m >= 25).  Around the second call
neither the device's free memory (cudaMemGetInfo) nor torch's allocated
bytes may change: the entry point allocates nothing once its first call on
the device has looked up the scratch array.  Sizes beyond the scratch are
rejected.  (The two-rank form is exercised in test_gpu_sharded.py.)  This file
is collected last so that a run stopping at the first failure has already run
every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
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


@pytest.mark.parametrize("m,f32", [(1, 0), (3, 0), (3, 1), (20, 0), (40, 0), (40, 1)])
def test_noalloc_matches_workspace_entry_point(dev, one_rank, m, f32):
    L = lib()
    n, k = 4096, 4096
    q = synth.unpack_codes_signed(synth.synth_codes(n, k, 880))
    s = synth.synth_scales(n, k, 880)
    w = import_planes(dev, q, s)
    dt = torch.float32 if f32 else torch.bfloat16
    iv = torch.int32 if f32 else torch.int16
    st = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # two calls in a row, different activations
        x = synth.synth_x(m, k, 881 + 10 * m + call)
        xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)
        ref = torch.empty((m, n), dtype=dt, device="cuda")
        ws = torch.empty((m, n), dtype=dt, device="cuda")
        check(L.xq4_linear_sharded(one_rank, w.handle, xd.data_ptr(), ref.data_ptr(), ws.data_ptr(), m, f32, st))
        got = torch.full((m, n), float("nan"), dtype=dt, device="cuda")
        torch.cuda.synchronize()
        free0, alloc0 = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
        check(L.xq4_linear_sharded_noalloc(one_rank, w.handle, xd.data_ptr(), got.data_ptr(), m, f32, st))
        torch.cuda.synchronize()
        free1, alloc1 = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
        if call == 1:  # the first call may have loaded the library's module on this device
            assert (free1, alloc1) == (free0, alloc0), ("device memory changed", free0 - free1, alloc1 - alloc0)
        assert torch.isfinite(got).all().item(), f"call {call}: output not fully written"
        assert torch.equal(got.view(iv), ref.view(iv)), f"call {call}: bits differ from xq4_linear_sharded"
        # and within the parity bars against the oracle (rows subset)
        rows = np.arange(0, n, 61)
        want = O.gemv_q(q[rows], s[rows], x) if m < 25 else O.gemv_bf16(O.dequant_planes(q[rows], s[rows]), x)
        a = got.float().cpu().numpy()[:, rows]
        if not f32:
            want = synth.bf16_bits_to_f32(O.round_bf16(want))
        max_rel, mae, _ = rel_metrics(a, want, f"no-alloc m={m} call {call}")
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
