"""Host mirror of the reference HAL's operator surface for the int4 path.

The reference drives its w4 GEMV through ``xnpu_hal`` (crates/xnpu-hal/src/
lib.rs:17-20): ``Device::open_default`` (accel.rs:122), ``BufferObject::new``
+ ``sync`` (bo.rs:42, :134), ``StartNpuCmd::new/arg64/submit`` (ert.rs:77-212)
and ``syncobj_timeline_wait`` (ert.rs:218).  This module offers the same
operations with the same meaning over libxq4 (include/xq4.h):

=========================================  =====================================
reference                                   here
=========================================  =====================================
Device::open_default / open                 Device.open_default() / Device.open(i)
Device::aie_metadata                        Device.metadata()
BufferObject::new(dev, ty, size)            BufferObject.new(dev, size)
mapping write + sync(ToDevice)              BufferObject.write(offset, data)
sync(FromDevice) + mapping read             BufferObject.read(offset, length)
BufferObject::xdna_addr                     BufferObject.device_ptr()
chain_tensor(W) over a w4_import .bin       Weight.import_(dev, src, LayoutDesc)
StartNpuCmd + arg64(W, x, C) + submit       LinearOp(w, x, y, m).submit(dev)
syncobj_timeline_wait(dev, sync, seq, ns)   timeline_wait(dev, seq, timeout_ns)
=========================================  =====================================

Errors raise :class:`Xq4Error` (an ``OSError`` carrying the XQ4_* status), as the
reference returns ``std::io::Result`` (crates/xnpu-hal/src/ioctl.rs:59-66);
a wait that passes its deadline raises with ``status == XQ4_ETIMEDOUT``.
"""
import ctypes

from . import _lib
from ._lib import (LayoutDesc, Xq4Error, check, lib, XQ4_LAYOUT_L1, XQ4_LAYOUT_L2,  # noqa: F401
                   XQ4_LAYOUT_PLANES, XQ4_CODE_S4, XQ4_CODE_U4_ZP8, XQ4_SCALE_BF16, XQ4_SCALE_FP16,
                   XQ4_OUT_BF16, XQ4_OUT_F32, XQ4_ETIMEDOUT)


def _buf_ptr(data):
    """(address, nbytes, keepalive) of a bytes-like / numpy array on the host."""
    try:
        import numpy as np
        if isinstance(data, np.ndarray):
            a = np.ascontiguousarray(data)
            return a.ctypes.data, a.nbytes, a
    except ImportError:
        pass
    mv = memoryview(data)
    if not mv.contiguous:
        raise ValueError("host data must be contiguous")
    if mv.readonly:
        b = (ctypes.c_char * mv.nbytes).from_buffer_copy(mv)
    else:
        b = (ctypes.c_char * mv.nbytes).from_buffer(mv)
    return ctypes.addressof(b), mv.nbytes, b


class Device:
    """One B200 with its in-order queue (the reference's Device + HwContext)."""

    def __init__(self, handle, ordinal):
        self._h = handle
        self.ordinal = ordinal

    @classmethod
    def open(cls, ordinal=0):
        h = ctypes.c_void_p()
        check(lib().xq4_device_open(ordinal, ctypes.byref(h)))
        return cls(h, ordinal)

    @classmethod
    def open_default(cls):
        return cls.open(0)

    @property
    def handle(self):
        if self._h is None:
            raise Xq4Error(_lib.XQ4_EINVAL, "device is closed")
        return self._h

    def metadata(self):
        info = _lib.DeviceInfo()
        check(lib().xq4_device_query(self.handle, ctypes.byref(info)))
        return {"ordinal": info.ordinal, "sm_count": info.sm_count,
                "cc": (info.cc_major, info.cc_minor), "hbm_bytes": info.hbm_bytes,
                "l2_bytes": info.l2_bytes, "name": info.name.decode()}

    def stream_handle(self):
        """The device queue as an integer cudaStream_t."""
        return lib().xq4_device_stream(self.handle) or 0

    def last_seq(self):
        return lib().xq4_last_seq(self.handle)

    def fault(self):
        """Read and clear the kernels' pipeline-fault bits (0 = none)."""
        bits = ctypes.c_uint32()
        check(lib().xq4_device_fault(self.handle, ctypes.byref(bits)))
        return bits.value

    def close(self):
        if self._h is not None:
            h, self._h = self._h, None
            check(lib().xq4_device_close(h))

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class BufferObject:
    """Device memory (the reference's BufferObject + its host mapping)."""

    def __init__(self, handle, dev):
        self._h = handle
        self.dev = dev

    @classmethod
    def new(cls, dev, size):
        h = ctypes.c_void_p()
        check(lib().xq4_buffer_create(dev.handle, size, ctypes.byref(h)))
        return cls(h, dev)

    @property
    def handle(self):
        if self._h is None:
            raise Xq4Error(_lib.XQ4_EINVAL, "buffer is destroyed")
        return self._h

    def size(self):
        return lib().xq4_buffer_size(self.handle)

    def device_ptr(self):
        return lib().xq4_buffer_device_ptr(self.handle)

    def write(self, offset, data):
        ptr, n, keep = _buf_ptr(data)
        check(lib().xq4_buffer_upload(self.handle, ptr, offset, n))
        del keep

    def read(self, offset, length):
        out = (ctypes.c_char * length)()
        check(lib().xq4_buffer_download(self.handle, ctypes.addressof(out), offset, length))
        return bytes(out)

    def destroy(self):
        if self._h is not None:
            h, self._h = self._h, None
            check(lib().xq4_buffer_destroy(h))

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


def layout_desc(layout, n, k, group=32, tsi=0, cols=0, code_format=XQ4_CODE_S4,
                scale_dtype=XQ4_SCALE_BF16, scale_offset=None, row_begin=0, row_end=0):
    """Build an xq4_layout_desc.  For PLANES the scale plane follows the code
    plane unless ``scale_offset`` says otherwise."""
    if scale_offset is None:
        scale_offset = n * k // 2 if layout == XQ4_LAYOUT_PLANES else 0
    return LayoutDesc(layout, n, k, group, tsi, cols, code_format, scale_dtype, scale_offset,
                      row_begin, row_end)


class Weight:
    """An int4 weight resident in HBM in the GPU layout."""

    def __init__(self, handle, dev):
        self._h = handle
        self.dev = dev
        n, k, nbytes = ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
        check(lib().xq4_weight_shape(handle, ctypes.byref(n), ctypes.byref(k), ctypes.byref(nbytes)))
        self.n, self.k, self.device_bytes = n.value, k.value, nbytes.value

    @classmethod
    def import_(cls, dev, src, desc):
        """Repack ``src`` (host bytes in ``desc.layout``) and upload it."""
        ptr, n, keep = _buf_ptr(src)
        h = ctypes.c_void_p()
        check(lib().xq4_weight_import(dev.handle, ptr, n, ctypes.byref(desc), ctypes.byref(h)))
        del keep
        return cls(h, dev)

    @property
    def handle(self):
        if self._h is None:
            raise Xq4Error(_lib.XQ4_EINVAL, "weight is destroyed")
        return self._h

    def destroy(self):
        if self._h is not None:
            h, self._h = self._h, None
            check(lib().xq4_weight_destroy(h))

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class LinearOp:
    """One w4 linear op with args [W, x, C] (the reference's StartNpuCmd)."""

    def __init__(self, weight, x_buf, y_buf, m, out_dtype=XQ4_OUT_BF16, x_off=0, y_off=0):
        self.weight, self.x_buf, self.y_buf = weight, x_buf, y_buf
        self.m, self.out_dtype, self.x_off, self.y_off = m, out_dtype, x_off, y_off

    def submit(self, dev):
        seq = ctypes.c_uint64()
        check(lib().xq4_linear(dev.handle, self.weight.handle, self.x_buf.handle, self.x_off,
                               self.y_buf.handle, self.y_off, self.m, self.out_dtype, ctypes.byref(seq)))
        return seq.value


class Chain:
    """A prebuilt chain of w4 linear ops run as one persistent kernel (the
    reference's chained op packets, built once and submitted together).

    ``ops`` is a list of (weight, x_ptr, y_ptr, m, out_dtype, wait_prev[,
    comm][, glue]) with raw device pointers (ints), an optional
    communicator handle for a column-sharded op and an optional dict of
    fused decode-step glue: {"norm_w": ptr, "eps": float, "residual": ptr,
    "swiglu": bool, "w4a8": bool}; see xq4_chain_create."""

    def __init__(self, dev, ops):
        arr = (_lib.ChainOp * len(ops))()
        for i, op in enumerate(ops):
            op = list(op)
            glue = op.pop() if isinstance(op[-1], dict) else {}
            w, xp, yp, m, od, wp = op[:6]
            comm = op[6] if len(op) > 6 else None
            arr[i] = _lib.ChainOp(w.handle, xp, yp, m, od, 1 if wp else 0, getattr(comm, "value", comm),
                                  glue.get("norm_w"), float(glue.get("eps", 1e-5)), glue.get("residual"),
                                  1 if glue.get("swiglu") else 0, 1 if glue.get("w4a8") else 0)
        h = ctypes.c_void_p()
        check(lib().xq4_chain_create(dev.handle, arr, len(ops), ctypes.byref(h)))
        self._h, self.dev, self.n_ops = h, dev, len(ops)
        self._keep = [op[0] for op in ops]  # the weights outlive the chain

    @property
    def handle(self):
        if not self._h:
            raise ValueError("chain destroyed")
        return self._h

    def submit(self):
        """On the device queue; returns the timeline point."""
        seq = ctypes.c_uint64()
        check(lib().xq4_chain_submit(self.dev.handle, self.handle, ctypes.byref(seq)))
        return seq.value

    def run(self, stream=None):
        """On the current torch stream (or ``stream``)."""
        check(lib().xq4_chain_run(self.handle, _torch_stream(stream)))

    def destroy(self):
        if self._h:
            lib().xq4_chain_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class Attention:
    """Decode attention of one token per layer (RoPE, per-head q/k RMSNorm,
    KV-cache append, GQA attention) on the device: the reference's decode
    glue (crates/xnpu-cli/src/main.rs:4817-4857, :4967-5033); see
    xq4_attn_decode."""

    def __init__(self, dev, heads, nkv, cache_seq, rope_base=10000.0):
        h = ctypes.c_void_p()
        check(lib().xq4_attn_create(dev.handle, heads, nkv, cache_seq, float(rope_base), ctypes.byref(h)))
        self._h, self.dev = h, dev
        self.heads, self.nkv, self.cache_seq = heads, nkv, cache_seq

    def decode(self, qkv, k_cache, v_cache, pos, out=None, q_norm=None, k_norm=None, stream=None):
        """qkv: CUDA bf16 [heads*128 + 2*nkv*128]; caches bf16 [nkv, cache_seq,
        128]; pos: CUDA int32 tensor of one element.  Returns out bf16
        [heads*128]."""
        import torch
        if out is None:
            out = torch.empty(self.heads * 128, dtype=torch.bfloat16, device=qkv.device)
        ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        check(lib().xq4_attn_decode(self._h, qkv.data_ptr(), ptr(q_norm), ptr(k_norm), k_cache.data_ptr(),
                                    v_cache.data_ptr(), pos.data_ptr(), out.data_ptr(), _torch_stream(stream)))
        return out

    def destroy(self):
        if self._h:
            lib().xq4_attn_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


def timeline_wait(dev, seq, timeout_ns):
    """Wait until op ``seq`` (and all before it) completed; raise on timeout."""
    check(lib().xq4_wait(dev.handle, seq, int(timeout_ns)))


# ---------------------------------------------------------------- torch glue
def _torch_stream(stream):
    import torch
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


def linear(weight, x, out_dtype=None, out=None, stream=None):
    """y = x @ dequant(W)^T for a torch CUDA tensor x of shape [m, k] (bf16).

    Runs on the current torch stream (or ``stream``).  ``out_dtype`` is
    torch.bfloat16 (default) or torch.float32."""
    import torch
    if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or x.shape[1] != weight.k:
        raise ValueError(f"x must be a CUDA bf16 tensor [m, {weight.k}]")
    x = x.contiguous()
    out_dtype = out_dtype or torch.bfloat16
    code = XQ4_OUT_F32 if out_dtype == torch.float32 else XQ4_OUT_BF16
    m = x.shape[0]
    if out is None:
        out = torch.empty((m, weight.n), dtype=out_dtype, device=x.device)
    check(lib().xq4_linear_raw(weight.handle, x.data_ptr(), out.data_ptr(), m, code, _torch_stream(stream)))
    return out


def quantize_x(x, stream=None):
    """W4A8 parity mode: int8 activations q [m, k] and bf16 group scales
    d [m, k/32] (as int16 bits) of a CUDA bf16 tensor x [m, k]."""
    import torch
    if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or x.shape[1] % 32:
        raise ValueError("x must be a CUDA bf16 tensor [m, k] with k a multiple of 32")
    x = x.contiguous()
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    d = torch.empty((m, k // 32), dtype=torch.int16, device=x.device)
    check(lib().xq4_quantize_x(x.data_ptr(), m, k, q.data_ptr(), d.data_ptr(), x.device.index or 0,
                               _torch_stream(stream)))
    return q, d


def linear_w4a8(weight, q, d, out_dtype=None, out=None, stream=None):
    """W4A8 parity mode: y = the reference's int8-activation GEMV of (q, d)
    from quantize_x against the weight."""
    import torch
    m = q.shape[0]
    out_dtype = out_dtype or torch.bfloat16
    code = XQ4_OUT_F32 if out_dtype == torch.float32 else XQ4_OUT_BF16
    if out is None:
        out = torch.empty((m, weight.n), dtype=out_dtype, device=q.device)
    check(lib().xq4_linear_w4a8(weight.handle, q.contiguous().data_ptr(), d.contiguous().data_ptr(),
                                out.data_ptr(), m, code, _torch_stream(stream)))
    return out


def dequant(weight, out=None, stream=None):
    """Dequantize the whole weight to a bf16 CUDA tensor [n, k]."""
    import torch
    if out is None:
        out = torch.empty((weight.n, weight.k), dtype=torch.bfloat16, device=f"cuda:{weight.dev.ordinal}")
    check(lib().xq4_dequant(weight.handle, out.data_ptr(), _torch_stream(stream)))
    return out


def gpu_layout_bytes(n, k):
    return lib().xq4_gpu_layout_bytes(n, k)


def repack_host(src, desc):
    """Repack on the host only (no device); returns the GPU-layout bytes."""
    import numpy as np
    r0, r1 = desc.row_begin, desc.row_end
    if r0 == 0 and r1 == 0:
        r1 = desc.n
    out = np.empty(max(gpu_layout_bytes(r1 - r0, desc.k), 1), dtype=np.uint8)
    ptr, n, keep = _buf_ptr(src)
    check(lib().xq4_repack_host(ptr, n, ctypes.byref(desc), out.ctypes.data, out.nbytes))
    del keep
    return out
