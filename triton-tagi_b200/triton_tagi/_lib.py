"""ctypes binding of libtagi_b200.so (the sm_100a CUDA library).

There is no fallback: if the library is missing or cannot be loaded, importing
any compute function raises, and every call checks the returned status and
raises ``ValueError`` (bad arguments) or ``RuntimeError`` (CUDA errors) with
the library's message.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("TAGI_B200_LIB", Path(__file__).resolve().parent / "libtagi_b200.so"))

_P, _I, _F, _D, _N, _Z, _U = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_double,
                              ctypes.c_int, ctypes.c_size_t, ctypes.c_uint64)
_CODES = {"p": _P, "i": _I, "f": _F, "d": _D, "n": _N, "z": _Z, "u": _U}

# name -> argument codes (stream last, always 'p'); returns int status unless listed in _RET.
_SIGS = {
    "tagi_fused_var_forward": "pppppp" + "iii" + "iiiiii" + "p",
    "tagi_moment_forward": "pp" + "iiii" + "ppi" + "pppp" + "iiii" + "iii" + "p",
    "tagi_fused_backward_delta": "ppppp" + "iii" + "iiiiii" + "p",
    "tagi_backward_delta_view": "pp" + "iiii" + "pi" + "pp" + "iiii" + "iii" + "p",
    "tagi_conv2d_backward_delta": "ppp" + "pp" + "iiiiiiiii" + "nn" + "pz" + "p",
    "tagi_linear_forward": "pppppp" + "pp" + "iii" + "pz" + "p",
    "tagi_linear_backward_delta": "ppp" + "pp" + "iii" + "pz" + "p",
    "tagi_conv2d_forward": "pppppp" + "pp" + "iiiiiiiii" + "n" + "pz" + "p",
    "tagi_nchw_to_nhwc": "pppp" + "iii" + "p",
    "tagi_fused_weight_grad_workspace_size": "iii",
    "tagi_store_workspace_size": "iii",
    "tagi_fused_weight_grad": "ppppp" + "iii" + "iiiiii" + "pz" + "p",
    "tagi_fused_weight_grad_static": "ppppp" + "iii" + "iiiiii" + "p",
    "tagi_param_grad_workspace_size": "iiin",
    "tagi_param_grad": "pipp" + "iiii" + "iii" + "nn" + "pppp" + "pppp" + "f" + "pz" + "p",
    "tagi_param_grad_t": "pipp" + "iiii" + "iii" + "nn" + "pppp" + "pppp" + "f" + "pz" + "p",
    "tagi_param_grad_bias_given": "pin" + "pp" + "iiii" + "iii" + "pn" + "pppp" + "pppp" + "f"
                                  + "pz" + "p",
    "tagi_apply_param_sums": "pp" + "ii" + "n" + "pppp" + "f" + "p",
    "tagi_bmm_tagi_var": "pppppp" + "iiii" + "iiiiiiiii" + "ff" + "p",
    "tagi_bmm_shared_right": "ppppp" + "iiii" + "iiiiiiiii" + "f" + "p",
    "tagi_bmm_shared_left": "ppppp" + "iiii" + "iiiiiiiii" + "f" + "p",
    "tagi_capped_update": "pppp" + "i" + "f" + "p",
    "tagi_innovation": "ppppp" + "i" + "f" + "p",
    "tagi_relu_forward": "ppppp" + "i" + "p",
    "tagi_jacobian_backward": "ppppp" + "i" + "p",
    "tagi_remax_forward": "ppppp" + "iii" + "p",
    "tagi_add_inplace": "pppp" + "i" + "p",
    "tagi_embedding_forward": "ppppp" + "iiii" + "p",
    "tagi_embedding_backward": "pppp" + "iiii" + "n" + "pp" + "p",
    "tagi_positional_add": "ppp" + "iii" + "p",
    "tagi_avgpool_forward": "pppp" + "iiiii" + "f" + "p",
    "tagi_avgpool_backward": "pppp" + "iiiii" + "f" + "p",
    "tagi_im2col": "pppp" + "iiiiiiii" + "p",
    "tagi_im2col_t": "pp" + "iiiiiiii" + "p",
    "tagi_col2im": "pppp" + "iiiiiiii" + "n" + "p",
    "tagi_bn_channel_sums": "ppp" + "iii" + "p",
    "tagi_bn_finalize": "p" + "i" + "d" + "ppppp" + "nn" + "ff" + "p",
    "tagi_bn_forward": "pppppppppppp" + "iii" + "f" + "p",
    "tagi_bn_train_forward": "ppppppppppppp" + "pp" + "iii" + "nn" + "ff" + "p",
    "tagi_bn_sync_forward": "ppp" + "d" + "p" * 13 + "iii" + "nn" + "ff" + "p",
    "tagi_bn_backward": "ppppppp" + "ppp" + "iii" + "f" + "ppp" + "f" + "p",
    "tagi_bn_apply_grads": "p" + "i" + "n" + "pppppppp" + "f" + "p",
    "tagi_rmsnorm_forward": "ppppppp" + "ii" + "f" + "p",
    "tagi_rmsnorm_backward": "pppppppp" + "ii" + "p",
    "tagi_apply_vector_sums": "pp" + "i" + "n" + "pppp" + "f" + "p",
    "tagi_version": "",
    "tagi_device_arch": "n",
    "tagi_last_error": "",
    "tagi_kernel_launches": "",
    "tagi_tma_launches": "",
    "tagi_tc_launches": "",
    "tagi_device_status": "n",
    "tagi_set_wait_limit_ns": "u",
    "tagi_peer_buffer_bytes": "ni",
    "tagi_peer_buffer_create": "zpp",
    "tagi_peer_buffer_open": "pp",
    "tagi_peer_buffer_close": "pn",
    "tagi_peer_allreduce_f64": "pipnnip" + "p",
    "tagi_peer_status": "n",
}
_RET = {
    "tagi_peer_buffer_bytes": _Z,
    "tagi_fused_weight_grad_workspace_size": _Z,
    "tagi_param_grad_workspace_size": _Z,
    "tagi_store_workspace_size": _Z,
    "tagi_last_error": ctypes.c_char_p,
    "tagi_kernel_launches": ctypes.c_uint64,
    "tagi_tma_launches": ctypes.c_uint64,
    "tagi_tc_launches": ctypes.c_uint64,
}

# Status codes (include/tagi_b200.h)
TAGI_OK, TAGI_E_BAD_ARG, TAGI_E_ALIGNMENT = 0, -1, -2
WGRAD_SUMS, WGRAD_DELTAS, WGRAD_UPDATE = 0, 1, 2


class _Lib:
    def __init__(self, path: Path):
        if not path.exists():
            raise ImportError(
                f"libtagi_b200.so not found at {path}; build it with "
                "`python triton-tagi_b200/build_lib.py` (nvcc, sm_100a)")
        self.path = path
        self.dll = ctypes.CDLL(str(path))
        self.fn = {}
        for name, codes in _SIGS.items():
            f = getattr(self.dll, name)
            f.argtypes = [_CODES[c] for c in codes]
            f.restype = _RET.get(name, ctypes.c_int)
            self.fn[name] = f

    hook = None  # optional callable(phase, name, args) used by the benchmark to time launches

    def __call__(self, name: str, *args):
        h = self.hook
        if h is not None:
            h("before", name, args)
        rc = self.fn[name](*args)
        if h is not None:
            h("after", name, args)
        if rc != 0:
            msg = self.fn["tagi_last_error"]().decode(errors="replace")
            if rc in (TAGI_E_BAD_ARG, TAGI_E_ALIGNMENT):
                raise ValueError(msg)
            raise RuntimeError(f"{name} failed ({rc}): {msg}")

    def size(self, name: str, *args) -> int:
        return int(self.fn[name](*args))


_instance: _Lib | None = None


def lib() -> _Lib:
    global _instance
    if _instance is None:
        _instance = _Lib(LIB_PATH)
    return _instance


def device_status(reset: bool = False) -> int:
    """0, or the code of a tensor-core kernel wait that timed out (synchronises)."""
    return int(lib().fn["tagi_device_status"](1 if reset else 0))


def check_device_status() -> None:
    """Raise RuntimeError if a tensor-core kernel wait or a peer exchange wait ran
    out since the last check (outputs are then incomplete); clears the words."""
    code = device_status(reset=True)
    if code != 0:
        raise RuntimeError(f"a tensor-core kernel gave up a tile (bounded wait {code} ran out); "
                           "its outputs are incomplete")
    if int(lib().fn["tagi_peer_status"](1)) != 0:
        raise RuntimeError("a peer-memory exchange wait ran out (a rank stopped?); the "
                           "statistics it carried were not reduced")


def set_wait_limit_ns(ns: int) -> None:
    """Limit of the tensor-core kernels' abortable waits (0 restores 2 s); a test hook."""
    rc = lib().fn["tagi_set_wait_limit_ns"](int(ns))
    if rc != 0:
        raise RuntimeError(lib().fn["tagi_last_error"]().decode(errors="replace"))


def kernel_launches() -> int:
    """Kernels launched by libtagi_b200 so far in this process."""
    return int(lib().fn["tagi_kernel_launches"]())


def tc_launches() -> int:
    """Of those, launches of the tcgen05 tensor-core contraction kernel."""
    return int(lib().fn["tagi_tc_launches"]())


def stream(t: torch.Tensor) -> int:
    """Raw cudaStream_t of the current torch stream on ``t``'s device."""
    return torch.cuda.current_stream(t.device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def check_cuda_f32(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("triton_tagi (B200) tensors must live on a CUDA device")
        if t.dtype != torch.float32:
            raise ValueError(f"expected float32 tensor, got {t.dtype}")


def workspace(nbytes: int, like: torch.Tensor) -> tuple[torch.Tensor | None, int | None, int]:
    """Scratch buffer for one call: returns (holder, pointer, bytes).

    The holder only has to live until the call has been enqueued: torch's
    caching allocator hands a freed block only to later work on the same
    stream, which runs after the kernels that used it."""
    if nbytes == 0:
        return None, None, 0
    buf = torch.empty(nbytes, dtype=torch.uint8, device=like.device)
    return buf, buf.data_ptr(), nbytes
