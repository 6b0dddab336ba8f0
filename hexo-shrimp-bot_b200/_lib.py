"""ctypes binding of ``libmantis_b200.so`` (the C ABI in include/mantis_b200.h).

The library is the product path: there is no CPU or Triton fallback. If it is
missing, or the device is not CUDA, every op raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libmantis_b200.so"

MB_F32, MB_BF16 = 0, 1
STATUS = {0: "OK", 1: "INVALID_ARGUMENT", 2: "LAUNCH_FAILED", 3: "TIMEOUT", 4: "UNSUPPORTED", 5: "DEVICE_ERROR"}
DEVICE_ERRORS = {1: "an index array held a value out of range", 2: "keys that must be sorted were not",
                 3: "a CSR run was malformed"}

# Argument codes: p pointer, i int32, l int64, f float.
SIGNATURES = {
    "mb_version": "",
    "mb_last_error": "",
    "mb_device_error": "ppi",
    "mb_csr_from_sorted": "pllpp",
    "mb_argsort_workspace": "lip",
    "mb_argsort": "plippplp",
    "mb_gather_i64": "plplpp",
    "mb_radius_class": "pppplpp",
    "mb_div_i64": "pllpp",
    "mb_run_reduce": "pillppllplplpilp",
    "mb_row_encode": "pilplppplpppilpilp",
    "mb_cell_pass": "pilplplpppplppip",
    "mb_cell_pass_noalloc": "pilplplpppplpip",
    "mb_segment_attention": "plpplilliiplpipppppilppp",
    "mb_segment_attention_grouped": "plpplilliiplpippppppllpilp",
    "mb_hex_message_pass": "pllpppplp",
    "mb_gemm_rows_ln": "pllppplfpppilpppilpppilp",
    "mb_axial_attention": "pppliillllpppplllp",
    "mb_radius_pack_edges": "ppppplllllpp",
    "mb_radius_read": "plppllliiplppppppppllpilp",
    "mb_radius_slots": "ppppplllpplp",
    "mb_radius_slots_size": "lllp",
    "mb_stone_attention_engine": "i",
    "mb_stone_attention": "pppiliilllplplipilllpp",
    "mb_window_latent_read": "plpplilliipppippp",
    "mb_window_latent_broadcast": "plpplilliippippp",
    "mb_latent_mix": "pppliliipip",
    "mb_segment_attention_backward": "pppilliiplpippppppplpppppppppppp",
    "mb_stone_attention_backward": "pppppiliilllplpppppp",
    "mb_window_latent_read_backward": "pppippppppplliipppp",
    "mb_window_latent_broadcast_backward": "pppipppppplliipppppp",
    "mb_row_encode_backward": "pilplppplpllppppppp",
    "mb_layer_norm": "pilpllppfpilp",
    "mb_add_ln": "plpilpllfpppilpppilpppilp",
    "mb_embed": "plpplpllpp",
    "mb_cell_init": "ppplppllpp",
    "mb_residual_add": "pilppilllp",
    "mb_add_gather": "pilpillpllip",
    "mb_tokens_gather": "ppppllpp",
    "mb_tokens_scatter_add": "ppppllpiip",
    "mb_latent_mean": "pllpp",
    "mb_value_head": "ppillpppplllppfpippippippppp",
    "mb_compose_q": "plplfppp",
    "mb_linear": "pilllpiplipilp",
    "mb_gemm_weight_image": "pllpp",
    "mb_gemm_rows": "pillppfppiplplp",
    "mb_gemm_rows_ex": "pilllppfplpiplplplp",
    "mb_gemm_rows_head": "pllplppllpppiplp",
    "mb_gemm_set_plan": "ii",
    "mb_encode_positions": "lpppppppip",
    "mb_encoding_sizes": "pp",
    "mb_encoding_fill": "ppi",
    "mb_encoding_fill_narrow": "ppi",
    "mb_encoding_free": "p",
    "mb_encoder_table": "ipl",
    "mb_segment_argmax": "ppllpp",
    "mb_klent_improve": "ppppllffpppppppppp",
}
_CT = {"p": ctypes.c_void_p, "i": ctypes.c_int, "l": ctypes.c_int64, "f": ctypes.c_float}

_lock = threading.Lock()
_lib = None


class MantisError(RuntimeError):
    pass


def load():
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise MantisError(
                    f"{LIB_PATH.name} is not built; run hexo-shrimp-bot_b200/build.py (nvcc, sm_100a)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, sig in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = [_CT[c] for c in sig]
                fn.restype = ctypes.c_int
            lib.mb_last_error.restype = ctypes.c_char_p
            _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


_calls = 0


def call_count() -> int:
    """Native entry-point calls so far (each launches the op's kernels)."""
    return _calls


def call(name: str, *args) -> None:
    global _calls
    lib = _lib or load()
    _calls += 1
    status = getattr(lib, name)(*args)
    if status != 0:
        msg = lib.mb_last_error().decode(errors="replace")
        kind = STATUS.get(status, str(status))
        if status == 1:
            raise ValueError(f"{name}: {msg}")
        raise MantisError(f"{name} failed ({kind}): {msg}")


def ptr(t):
    """Device pointer of a tensor (None for None)."""
    if t is None:
        return None
    return t.data_ptr()


def stream_of(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return MB_F32
    if dt == torch.bfloat16:
        return MB_BF16
    raise ValueError(f"unsupported dtype {dt}; the kernels take float32 or bfloat16")


def check_device_error(device=None, clear: bool = True) -> None:
    """Raise ValueError if a kernel recorded an out-of-range index (syncs)."""
    code = ctypes.c_uint32(0)
    call("mb_device_error", stream_of(device), ctypes.byref(code), int(clear))
    if code.value:
        raise ValueError(f"device-side validation failed: {DEVICE_ERRORS.get(code.value, code.value)}")
