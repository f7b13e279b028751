"""Device guards of the kernel layer.

The reference guards its device path with ``require_npu`` /
``import_torch_npu`` (core/runtime.py:36-79); here the device path is
libqkv_sm100 on a CUDA sm_100 GPU, and the guard fails closed with the same
style of message when that is not available.
"""

from __future__ import annotations

import importlib


def cuda_sm100_available() -> bool:
    try:
        torch = importlib.import_module("torch")
    except ImportError:
        return False
    try:
        if not torch.cuda.is_available():
            return False
        major, _ = torch.cuda.get_device_capability()
        return major == 10
    except Exception:
        return False


def require_cuda_sm100(what: str) -> None:
    if not cuda_sm100_available():
        raise RuntimeError(
            f"{what} requires an NVIDIA Blackwell (sm_100) GPU, but none is "
            "available. The quantized-KV kernel layer targets sm_100a only; the "
            "layout contract and host bookkeeping work on any machine."
        )


def import_torch(what: str = "this code path"):
    try:
        return importlib.import_module("torch")
    except ImportError as exc:
        raise RuntimeError(f"{what} requires torch, which is not installed") from exc


__all__ = ["cuda_sm100_available", "import_torch", "require_cuda_sm100"]
