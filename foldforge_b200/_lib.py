"""ctypes binding of the C ABI (``include/foldforge_b200.h``) in ``_ffb.so``.

The library is required: there is no fallback implementation behind these bindings. A
missing or unloadable library raises :class:`LibraryMissing` at the first call.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIBRARY = Path(os.environ.get("FFB_LIBRARY", _HERE / "_ffb.so"))

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_i64 = ctypes.c_int64
c_float = ctypes.c_float

#: name -> argument types, exactly as declared in include/foldforge_b200.h
SIGNATURES: dict[str, list] = {
    "ffb_version": [],
    "ffb_last_error": [],
    "ffb_device_error": [ctypes.POINTER(c_int), c_void_p],
    "ffb_layernorm_fwd": [c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_int, c_float, c_int, c_void_p],
    "ffb_gemm_bf16_nt": [
        c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
        c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
    ],
    "ffb_trimul_packed_bytes": [],
    "ffb_trimul_workspace_bytes": [c_int, c_int],
    "ffb_trimul_prepare": [c_void_p] * 12,
    "ffb_trimul_fwd": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_int, c_int, c_int,
                       c_int, c_void_p],
    "ffb_trimul_fwd_stages": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_int, c_int,
                              c_int, c_int, c_int, c_void_p],
    "ffb_triattn_fwd_stages": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_int, c_int,
                               c_int, c_int, c_int, c_void_p],
    "ffb_triattn_packed_bytes": [],
    "ffb_triattn_workspace_bytes": [c_int, c_int],
    "ffb_triattn_prepare": [c_void_p] * 10,
    "ffb_triattn_fwd": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_int, c_int, c_int,
                        c_int, c_void_p],
    "ffb_transition_packed_bytes": [],
    "ffb_transition_prepare": [c_void_p] * 7,
    "ffb_transition_fwd": [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p],
    "ffb_apb_packed_bytes": [],
    "ffb_apb_workspace_bytes": [c_int, c_int],
    "ffb_apb_prepare": [c_void_p] * 12,
    "ffb_apb_fwd": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_float, c_void_p, c_void_p,
                    ctypes.c_size_t, c_int, c_int, c_int, c_void_p],
    "ffb_single_transition_packed_bytes": [],
    "ffb_single_transition_workspace_bytes": [c_int, c_int],
    "ffb_single_transition_prepare": [c_void_p] * 7,
    "ffb_single_transition_fwd_noalloc": [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p],
    "ffb_single_transition_fwd": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_int, c_int,
                                  c_int, c_void_p],
    # row-sharded pieces (B = 1)
    "ffb_trimul_shard_proj": [c_void_p] * 6 + [c_int, c_int, c_int, c_void_p],
    "ffb_trimul_shard_contract": [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p],
    "ffb_trimul_shard_out": [c_void_p] * 7 + [c_int, c_int, c_int, c_int, c_void_p],
    "ffb_triattn_shard_proj": [c_void_p] * 6 + [c_int, c_int, c_void_p],
    "ffb_triattn_shard_attn": [c_void_p] * 6 + [c_int, c_int, c_int, c_void_p],
    "ffb_triattn_shard_out": [c_void_p] * 5 + [c_int, c_int, c_int, c_int, c_void_p],
    "ffb_transition_shard_fwd": [c_void_p] * 4 + [c_int, c_int, c_int, c_int, c_void_p],
    "ffb_apb_shard_pair_bias": [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p],
    "ffb_apb_single_workspace_bytes": [c_int],
    "ffb_apb_shard_single": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_float, c_void_p, c_void_p,
                             ctypes.c_size_t, c_int, c_int, c_void_p],
    "ffb_apb_shard_single_rows": [c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p, ctypes.c_size_t,
                                  c_int, c_int, c_int, c_int, c_void_p],
    # token diffusion transformer block
    "ffb_dit_packed_bytes": [],
    "ffb_dit_prepare": [c_void_p, c_void_p, c_void_p],
    "ffb_dit_tables_bytes": [c_int],
    "ffb_dit_condition_workspace_bytes": [c_int],
    "ffb_dit_condition": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_int, c_void_p],
    "ffb_dit_workspace_bytes": [c_int, c_int],
    "ffb_dit_fwd": [c_void_p] * 6 + [ctypes.c_size_t, c_int, c_int, c_void_p],
    # row-shard exchanges over NVLink peer memory (CUDA IPC buffers)
    "ffb_p2p_handle_bytes": [],
    "ffb_p2p_alloc": [ctypes.c_size_t, ctypes.POINTER(c_void_p), c_void_p],
    "ffb_p2p_open": [c_void_p, ctypes.POINTER(c_void_p)],
    "ffb_p2p_close": [c_void_p],
    "ffb_p2p_free": [c_void_p],
    "ffb_shard_transpose_p2p": [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p],
    "ffb_shard_gather_p2p": [c_void_p, ctypes.c_size_t, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p],
    "ffb_shard_wait_p2p": [c_void_p, c_void_p, c_int, c_i64, c_void_p],
    "ffb_shard_rows_p2p": [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p],
    "ffb_trimul_channel_contract": [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p],
    # fp32 / any-width path (FP32 SIMT kernels)
    "ffb_trimul_f32_workspace_bytes": [c_int, c_int, c_int, c_int],
    "ffb_trimul_fwd_f32": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_int, c_int, c_int,
                           c_int, c_int, c_int, c_void_p],
    "ffb_triattn_f32_workspace_bytes": [c_int, c_int, c_int, c_int, c_int],
    "ffb_triattn_fwd_f32": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_int, c_int, c_int,
                            c_int, c_int, c_int, c_int, c_void_p],
    "ffb_transition_f32_workspace_bytes": [c_i64, c_int, c_int],
    "ffb_transition_fwd_f32": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_int, c_int,
                               c_int, c_int, c_int, c_int, c_void_p],
    "ffb_apb_f32_workspace_bytes": [c_int, c_int, c_int, c_int, c_int],
    "ffb_apb_fwd_f32": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p,
                        ctypes.c_size_t, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p],
    # MSA module
    "ffb_opm_packed_bytes": [],
    "ffb_opm_workspace_bytes": [c_int, c_int],
    "ffb_opm_prepare": [c_void_p] * 8,
    "ffb_opm_fwd": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_int, c_int, c_int, c_float,
                    c_void_p],
    "ffb_pwa_packed_bytes": [],
    "ffb_pwa_workspace_bytes": [c_int, c_int],
    "ffb_pwa_prepare": [c_void_p] * 9,
    "ffb_pwa_fwd": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_int, c_int, c_int,
                    c_void_p],
    "ffb_transition_gemm_packed_bytes": [c_int, c_int],
    "ffb_transition_gemm_workspace_bytes": [c_i64, c_int, c_int],
    "ffb_transition_gemm_prepare": [c_void_p] * 5 + [c_int, c_int, c_void_p, c_void_p],
    "ffb_transition_gemm_fwd": [c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_size_t, c_i64, c_int, c_int,
                                c_void_p],
}

#: entry points that return a size_t instead of a status
SIZE_RESULT = {"ffb_apb_packed_bytes", "ffb_apb_workspace_bytes", "ffb_single_transition_packed_bytes",
               "ffb_single_transition_workspace_bytes", "ffb_transition_packed_bytes", "ffb_trimul_packed_bytes",
               "ffb_trimul_workspace_bytes", "ffb_triattn_packed_bytes", "ffb_triattn_workspace_bytes",
               "ffb_dit_packed_bytes", "ffb_dit_tables_bytes", "ffb_dit_condition_workspace_bytes", "ffb_dit_workspace_bytes",
               "ffb_apb_single_workspace_bytes", "ffb_trimul_f32_workspace_bytes", "ffb_triattn_f32_workspace_bytes",
               "ffb_transition_f32_workspace_bytes", "ffb_apb_f32_workspace_bytes", "ffb_opm_packed_bytes",
               "ffb_opm_workspace_bytes", "ffb_pwa_packed_bytes", "ffb_pwa_workspace_bytes",
               "ffb_transition_gemm_packed_bytes", "ffb_transition_gemm_workspace_bytes"}

STATUS = {0: "FFB_OK", 1: "FFB_ERR_ARG", 2: "FFB_ERR_UNSUPPORTED", 3: "FFB_ERR_CUDA", 4: "FFB_ERR_DEVICE"}


class LibraryMissing(RuntimeError):
    """The compiled sm_100a library could not be loaded."""


class KernelError(RuntimeError):
    """A C-ABI entry point returned a non-OK status."""

    def __init__(self, fn: str, status: int, message: str) -> None:
        super().__init__(f"{fn}: {STATUS.get(status, status)}: {message}")
        self.status = status


class UnsupportedCall(KernelError):
    """FFB_ERR_UNSUPPORTED: the call is outside the kernels' range."""


_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """The loaded library (loaded once; raises :class:`LibraryMissing`)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIBRARY.exists():
        raise LibraryMissing(f"{LIBRARY} is not built; run `python -m foldforge_b200.csrc.build`")
    try:
        lib = ctypes.CDLL(str(LIBRARY))
    except OSError as exc:  # pragma: no cover - depends on the machine
        raise LibraryMissing(f"cannot load {LIBRARY}: {exc}") from exc
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        if name == "ffb_last_error":
            fn.restype = ctypes.c_char_p
        elif name in SIZE_RESULT:
            fn.restype = ctypes.c_size_t
        else:
            fn.restype = c_int
    _lib = lib
    return lib


#: kernels each forward entry point launches (the bench's count of this library's launches)
LAUNCHES = {
    "ffb_layernorm_fwd": 1, "ffb_gemm_bf16_nt": 1, "ffb_trimul_fwd": 3, "ffb_triattn_fwd": 3,
    "ffb_transition_fwd": 1, "ffb_apb_fwd": 5, "ffb_single_transition_fwd": 3,
    "ffb_trimul_shard_proj": 1, "ffb_trimul_shard_contract": 1, "ffb_trimul_shard_out": 1,
    "ffb_triattn_shard_proj": 1, "ffb_triattn_shard_attn": 1, "ffb_triattn_shard_out": 1,
    "ffb_transition_shard_fwd": 1, "ffb_apb_shard_pair_bias": 1, "ffb_apb_shard_single": 4, "ffb_apb_shard_single_rows": 4, "ffb_dit_prepare": 17, "ffb_dit_condition": 6, "ffb_dit_fwd": 7,
    "ffb_single_transition_fwd_noalloc": 3,
    "ffb_shard_transpose_p2p": 1, "ffb_shard_gather_p2p": 1, "ffb_shard_wait_p2p": 1, "ffb_shard_rows_p2p": 1,
    "ffb_trimul_channel_contract": 1,
    "ffb_trimul_fwd_f32": 12, "ffb_triattn_fwd_f32": 8, "ffb_transition_fwd_f32": 5, "ffb_apb_fwd_f32": 9,
    "ffb_opm_fwd": 6, "ffb_pwa_fwd": 8, "ffb_transition_gemm_fwd": 3,
}
launch_count = 0


def _stage_launches(name: str, args) -> int:
    return bin(int(args[10])).count("1")


def call(name: str, *args) -> None:
    """Call an entry point; raise on a non-OK status."""
    global launch_count
    lib = load()
    status = getattr(lib, name)(*args)
    if status == 0:
        if name in ("ffb_trimul_fwd_stages", "ffb_triattn_fwd_stages"):
            launch_count += _stage_launches(name, args)
        else:
            launch_count += LAUNCHES.get(name, 0)
    if status != 0:
        msg = lib.ffb_last_error().decode(errors="replace")
        cls = UnsupportedCall if status == 2 else KernelError
        raise cls(name, status, msg)


def device_error(stream: int = 0) -> int:
    """Synchronise ``stream`` and return (and clear) the device error word (0 = none)."""
    lib = load()
    code = c_int(0)
    status = lib.ffb_device_error(ctypes.byref(code), c_void_p(stream))
    if status not in (0, 4):
        raise KernelError("ffb_device_error", status, lib.ffb_last_error().decode(errors="replace"))
    return code.value
