"""Small torch <-> C-ABI helpers shared by the op wrappers."""

from __future__ import annotations

import torch

from . import _lib


def require_cuda(what: str, *tensors: torch.Tensor) -> None:
    """The kernels run on CUDA tensors only; anything else is an error, never a
    silent CPU fallback."""
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(
                f"{what} runs on the B200 kernels of libqkv_sm100 and needs CUDA "
                f"tensors, got a tensor on {t.device}"
            )


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# the current stream's raw handle without building a torch.cuda.Stream object
# (microseconds per call on the decode step's host path); the public API is
# the fallback
_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: torch.device) -> int:
    if _RAW_STREAM is not None:
        return _RAW_STREAM(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


_DTYPE = {torch.float32: _lib.QKV_F32, torch.bfloat16: _lib.QKV_BF16, torch.float16: _lib.QKV_F16}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE[t.dtype]
    except KeyError:
        raise RuntimeError(f"unsupported floating dtype {t.dtype}; expected float32/bfloat16/float16") from None


def index_code(t: torch.Tensor) -> int:
    if t.dtype == torch.int64:
        return _lib.QKV_I64
    if t.dtype == torch.int32:
        return _lib.QKV_I32
    raise RuntimeError(f"index tensors must be int32/int64, got {t.dtype}")


class Workspace:
    """Per-device scratch buffer for split-KV partials, grown on demand and
    reused across calls on the same stream order."""

    def __init__(self) -> None:
        self._bufs: dict[int, torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor | None:
        if nbytes <= 0:
            return None
        idx = device.index if device.index is not None else torch.cuda.current_device()
        buf = self._bufs.get(idx)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            self._bufs[idx] = buf
        return buf


WORKSPACE = Workspace()
