"""B200-native (sm_100a) fused attention forward, behind the reference's launch API.

Python mirror of the C++ API a caller of RichterWang/cuda_fused_attention uses
(include/flash_attention.h, namespace cuda_op_lab::flash_attention): an
AttentionShape, default_scale, attention_flops, and the four-function pattern
of a kernel variant (supported / launch / query / hbm_bytes). Every compute
call goes through the C ABI of include/fa_sm100.h in libfa_sm100.so; PyTorch is
used only to hold device memory and streams.

    from cuda_fused_attention_b200 import AttentionShape, launch_attention_sm100
    launch_attention_sm100(q, k, v, o, AttentionShape(1, 2, 128, 64), causal=False)
"""
import ctypes
from dataclasses import dataclass

from . import _lib
from ._lib import (STATUS_OK, STATUS_INVALID_ARGUMENT, STATUS_UNSUPPORTED, STATUS_MISALIGNED,
                   STATUS_NO_SM100, STATUS_DEVICE_TIMEOUT, FaTilingInfo)

__all__ = [
    "AttentionShape", "FaError", "default_scale", "attention_flops", "sm100_supported",
    "launch_attention_sm100", "launch_attention_sm100_slabs", "query_sm100", "sm100_hbm_bytes",
    "sm100_min_bytes", "attention_forward", "attention_forward_host", "device_status",
    "STATUS_OK", "STATUS_INVALID_ARGUMENT", "STATUS_UNSUPPORTED", "STATUS_MISALIGNED",
    "STATUS_NO_SM100", "STATUS_DEVICE_TIMEOUT",
]


@dataclass(frozen=True)
class AttentionShape:
    """include/flash_attention.h:12-18: self-attention, seq_len queries and keys."""
    batch: int
    heads: int
    seq_len: int
    head_dim: int

    @property
    def slabs(self):
        return self.batch * self.heads

    @property
    def numel(self):
        return self.batch * self.heads * self.seq_len * self.head_dim


class FaError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, status, what=""):
        self.status = int(status)
        text = _lib.load().fa_sm100_status_string(self.status).decode()
        super().__init__(f"{what}: status {self.status} ({text})" if what else f"status {self.status} ({text})")


def _check(status, what):
    if status != STATUS_OK:
        raise FaError(status, what)


def default_scale(head_dim):
    """include/flash_attention.h:21-24 (float32 1/sqrt(D))."""
    return float(_lib.load().fa_default_scale(int(head_dim)))


def attention_flops(shape, causal):
    """kernels/v0_unfused.cu:118-126: 4*B*H*D*pairs, pairs N^2 or N(N+1)/2."""
    return float(_lib.load().fa_attention_flops(shape.batch, shape.heads, shape.seq_len, shape.head_dim,
                                                 1 if causal else 0))


def sm100_supported(head_dim):
    """Counterpart of tensorcore_v3_supported (include/flash_attention.h:90)."""
    return bool(_lib.load().fa_sm100_supported(int(head_dim)))


def query_sm100(head_dim):
    """Counterpart of query_tensorcore_v3 (include/flash_attention.h:94); needs a GPU."""
    info = FaTilingInfo()
    _check(_lib.load().fa_sm100_query(int(head_dim), ctypes.byref(info)), "fa_sm100_query")
    return {name: getattr(info, name) for name, _ in FaTilingInfo._fields_}


def sm100_hbm_bytes(shape, causal):
    """Counterpart of tensorcore_v3_hbm_bytes (include/flash_attention.h:96)."""
    return float(_lib.load().fa_sm100_hbm_bytes(shape.batch, shape.heads, shape.seq_len, shape.head_dim,
                                                 1 if causal else 0))


def sm100_min_bytes(shape):
    """Q, K, V read once and O written once."""
    return float(_lib.load().fa_sm100_min_bytes(shape.batch, shape.heads, shape.seq_len, shape.head_dim))


def _ptr(x):
    if isinstance(x, int):
        return x
    return int(x.data_ptr())


def _stream_handle(stream, like):
    if stream is None:
        import torch
        if hasattr(like, "device") and getattr(like.device, "type", None) == "cuda":
            return int(torch.cuda.current_stream(like.device).cuda_stream)
        return 0
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


def _check_tensor(name, t, shape):
    if isinstance(t, int):
        return
    import torch
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be bfloat16, got {t.dtype}")
    if not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous [batch, heads, seq_len, head_dim]")
    if t.numel() != shape.numel:
        raise ValueError(f"{name} has {t.numel()} elements, shape needs {shape.numel}")


def _device_of(*tensors):
    """The one CUDA device of the tensor arguments (None if all are raw pointers)."""
    devices = {t.device for t in tensors if not isinstance(t, int)}
    if len(devices) > 1:
        raise ValueError(f"q, k, v and o must be on one device, got {sorted(str(d) for d in devices)}")
    return devices.pop() if devices else None


def _on_device(device):
    """Make `device` current for the call: the C entry points launch on the current device."""
    import contextlib
    if device is None:
        return contextlib.nullcontext()
    import torch
    return torch.cuda.device(device)


def launch_attention_sm100(q, k, v, o, shape, causal=False, stream=None):
    """Counterpart of launch_attention_tensorcore_v3 (include/flash_attention.h:92).

    q, k, v, o: contiguous bf16 CUDA tensors (or raw device pointers) of
    shape.numel elements. Asynchronous on `stream` (default: torch's current
    stream of q's device). Raises FaError on a rejected argument or launch.
    """
    for name, t in (("q", q), ("k", k), ("v", v), ("o", o)):
        _check_tensor(name, t, shape)
    with _on_device(_device_of(q, k, v, o)):
        status = _lib.load().fa_sm100_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(o), shape.batch, shape.heads,
                                          shape.seq_len, shape.head_dim, 1 if causal else 0,
                                          _stream_handle(stream, q))
    _check(status, "fa_sm100_fwd")


def launch_attention_sm100_slabs(q, k, v, o, shape, causal, slab_begin, slab_end, stream=None):
    """Forward over slabs [slab_begin, slab_end) of batch*heads (one GPU's shard)."""
    for name, t in (("q", q), ("k", k), ("v", v), ("o", o)):
        _check_tensor(name, t, shape)
    with _on_device(_device_of(q, k, v, o)):
        status = _lib.load().fa_sm100_fwd_slabs(_ptr(q), _ptr(k), _ptr(v), _ptr(o), shape.batch, shape.heads,
                                                shape.seq_len, shape.head_dim, 1 if causal else 0,
                                                int(slab_begin), int(slab_end), _stream_handle(stream, q))
    _check(status, "fa_sm100_fwd_slabs")


def attention_forward(q, k, v, causal=False, stream=None):
    """Allocate O like q and run the forward pass; q/k/v are [B, H, N, D] bf16 CUDA tensors."""
    import torch
    if q.dim() != 4:
        raise ValueError("q must be [batch, heads, seq_len, head_dim]")
    shape = AttentionShape(*[int(x) for x in q.shape])
    o = torch.empty_like(q)
    launch_attention_sm100(q, k, v, o, shape, causal, stream)
    return o


def attention_forward_host(q, k, v, o, shape, causal=False):
    """End-to-end call with host buffers (fa_sm100_fwd_host): H2D, forward, D2H, synchronised.

    q, k, v, o are host arrays (torch CPU tensors or numpy arrays of bf16 bits);
    pinned memory gives overlapped copies.
    """
    def addr(x):
        if hasattr(x, "data_ptr"):
            return int(x.data_ptr())
        return int(x.ctypes.data)
    status = _lib.load().fa_sm100_fwd_host(addr(q), addr(k), addr(v), addr(o), shape.batch, shape.heads,
                                           shape.seq_len, shape.head_dim, 1 if causal else 0)
    _check(status, "fa_sm100_fwd_host")


def device_status():
    """Synchronise the current device and read+clear the kernel's error word: (status, raw word)."""
    word = ctypes.c_uint(0)
    status = _lib.load().fa_sm100_device_status(ctypes.byref(word))
    return int(status), int(word.value)
