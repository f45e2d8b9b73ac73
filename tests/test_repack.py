"""Host repacker (libxq4.so, no GPU needed): reference layouts -> GPU layout,
checked bit-exactly against the oracle through an independent numpy decoder."""
import json

import numpy as np
import pytest

from oracle import oracle as O
from xnpu_b200 import hal, synth
from xnpu_b200._lib import Xq4Error, XQ4_EINVAL
import xq4g_ref


def planes(n, k, seed):
    codes = synth.synth_codes(n, k, seed)
    return synth.unpack_codes_signed(codes), synth.synth_scales(n, k, seed), codes


def check_decoded(img, q, s):
    n, k = q.shape
    dq, ds, qp, sp = xq4g_ref.decode(img, n, k)
    assert np.array_equal(dq, q)
    assert np.array_equal(ds, s)
    # padding is q = 0 with scale 0
    assert not qp[n:].any() and not qp[:, k:].any()
    assert not sp[n:].any() and not sp[:, -(-k // 32):].any()
    # dequantized values are the oracle's, bit for bit
    assert np.array_equal(O.dequant_planes(dq, ds), O.dequant_planes(q, s))


@pytest.mark.parametrize("n,k,tsi", [(128, 2048, 16), (256, 4096, 4), (128, 6144, 16)])
def test_repack_l1(n, k, tsi):
    q, s, _ = planes(n, k, 11)
    pack = O.l1_pack(q, s, tsi=tsi)
    img = hal.repack_host(pack, hal.layout_desc(hal.XQ4_LAYOUT_L1, n, k, tsi=tsi, cols=8))
    assert img.size == hal.gpu_layout_bytes(n, k)
    check_decoded(img, q, s)


@pytest.mark.parametrize("n,k", [(128, 2048), (256, 4096), (128, 6144)])
def test_repack_l2(n, k):
    q, s, _ = planes(n, k, 12)
    pack = O.l2_pack(q, s)
    img = hal.repack_host(pack, hal.layout_desc(hal.XQ4_LAYOUT_L2, n, k))
    check_decoded(img, q, s)


def test_repack_fixture_layouts_agree(golden_dir):
    """The committed L1 and L2 images of one matrix repack to the same bytes."""
    man = json.loads((golden_dir / "manifest.json").read_text())["layouts"]
    m, k = man["m"], man["k"]
    l1 = np.fromfile(golden_dir / "l1_small.bin", dtype=np.uint8)
    l2 = np.fromfile(golden_dir / "l2_small.bin", dtype=np.uint8)
    a = hal.repack_host(l1, hal.layout_desc(hal.XQ4_LAYOUT_L1, m, k, tsi=16, cols=8))
    b = hal.repack_host(l2, hal.layout_desc(hal.XQ4_LAYOUT_L2, m, k))
    assert np.array_equal(a, b)
    q = synth.unpack_codes_signed(synth.synth_codes(m, k, man["seed"]))
    check_decoded(a, q, synth.synth_scales(m, k, man["seed"]))


@pytest.mark.parametrize("n,k", [(1, 32), (17, 96), (100, 4096), (333, 160)])
def test_repack_planes_ragged(n, k):
    """Rows not a multiple of 16 and K not a multiple of 64 are zero-padded."""
    q, s, codes = planes(n, k, 13)
    img = hal.repack_host(synth.planes_bytes(codes, s), hal.layout_desc(hal.XQ4_LAYOUT_PLANES, n, k))
    check_decoded(img, q, s)


def test_repack_planes_u4_and_fp16():
    n, k = 64, 256
    q, s, codes = planes(n, k, 14)
    u4 = codes ^ np.uint8(0x88)  # zero-point-8 codes
    s16 = synth.bf16_bits_to_f32(s).astype(np.float16).view(np.uint16)  # exact by construction
    img = hal.repack_host(synth.planes_bytes(u4, s16),
                          hal.layout_desc(hal.XQ4_LAYOUT_PLANES, n, k, code_format=hal.XQ4_CODE_U4_ZP8,
                                          scale_dtype=hal.XQ4_SCALE_FP16))
    check_decoded(img, q, s)


def test_repack_row_range_is_a_shard():
    n, k = 256, 2048
    q, s, _ = planes(n, k, 15)
    pack = O.l1_pack(q, s, tsi=16)
    for r0, r1 in [(0, 64), (64, 128), (128, 256), (40, 100)]:
        img = hal.repack_host(pack, hal.layout_desc(hal.XQ4_LAYOUT_L1, n, k, tsi=16, cols=8,
                                                    row_begin=r0, row_end=r1))
        check_decoded(img, q[r0:r1], s[r0:r1])


def _expect_einval(src, desc, text):
    with pytest.raises(Xq4Error) as ei:
        hal.repack_host(src, desc)
    assert ei.value.status == XQ4_EINVAL
    assert text in str(ei.value)


def test_repack_rejects_bad_input():
    q, s, codes = planes(128, 2048, 16)
    pack = O.l1_pack(q, s, tsi=16)
    L1 = hal.XQ4_LAYOUT_L1
    _expect_einval(pack, hal.layout_desc(L1, 128, 2048, group=64, tsi=16, cols=8), "group must be 32")
    _expect_einval(pack, hal.layout_desc(L1, 128, 2048, tsi=48, cols=8), "L1 geometry")
    _expect_einval(pack[:-1], hal.layout_desc(L1, 128, 2048, tsi=16, cols=8), "stale import")
    _expect_einval(pack, hal.layout_desc(L1, 128, 2048, tsi=16, cols=8, row_begin=10, row_end=5), "row range")
    _expect_einval(pack, hal.layout_desc(hal.XQ4_LAYOUT_L2, 128, 1024), "L2 geometry")
    _expect_einval(pack, hal.layout_desc(99, 128, 2048), "unknown layout")
    bad16 = np.full(128 * 64, 0x3C01, dtype=np.uint16)  # 1 + 2^-10: not a bf16 value
    _expect_einval(synth.planes_bytes(codes, bad16.reshape(128, 64)),
                   hal.layout_desc(hal.XQ4_LAYOUT_PLANES, 128, 2048, scale_dtype=hal.XQ4_SCALE_FP16),
                   "not exactly representable")
