"""ctypes binding of libb2p.so (the C ABI declared in include/b2p.h).

Loading fails loudly: there is no CPU or PyTorch fallback for any entry point.
Signatures are declared once here; `ABI` maps each exported name to its
(restype, argtypes).
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
LIB_PATH = PKG / "libb2p.so"
HEADER_DIR = ROOT / "include"

vp = C.c_void_p
i32 = C.c_int
i64 = C.c_longlong
u64 = C.c_uint64
f32 = C.c_float
fp = C.POINTER(C.c_float)
ip = C.POINTER(C.c_int)
u16p = C.POINTER(C.c_uint16)
u64p = C.POINTER(C.c_uint64)
szt = C.c_size_t
cstr = C.c_char_p

# name -> (restype, [argtypes])
ABI: dict[str, tuple] = {
    "b2p_init": (i32, [i32]),
    "b2p_last_error": (cstr, []),
    "b2p_version": (cstr, []),
    "b2p_device_status": (i32, [vp]),
    "b2p_gemm": (i32, [vp, vp, vp, i32, i32, i32, i32, i32, i32, vp]),
    "b2p_attention": (i32, [vp, i32, vp, i32, vp, i32, i32, i32, i32, i32, vp]),
    "b2p_attention_backward": (i32, [vp, i32, vp, vp, i32, vp, vp, i32, i32, i32, i32, i32, f32, i32, vp]),
    "b2p_model_create": (vp, [vp]),
    "b2p_model_free": (None, [vp]),
    "b2p_model_trainable_count": (i64, [vp]),
    "b2p_model_stream": (vp, [vp]),
    "b2p_model_set_layer": (i32, [vp, i32, fp, fp, fp, fp, fp, fp, fp]),
    "b2p_model_set_embedding": (i32, [vp, fp, ip, i32]),
    "b2p_model_set_trainable": (i32, [vp, vp, i64]),
    "b2p_model_get_trainable": (i32, [vp, vp, i64]),
    "b2p_model_eval": (i32, [vp, u16p, u16p, i32, vp, i32, fp]),
    "b2p_model_group_losses": (i32, [vp, vp, i32]),
    "b2p_mezo_step": (i32, [vp, u16p, u16p, u64, f32, f32, fp, fp, fp]),
    "b2p_mezo_eval": (i32, [vp, u16p, u16p, i32, u64p, i32, f32, vp]),
    "b2p_mezo_update": (i32, [vp, u64p, vp, i32, f32, f32]),
    "b2p_model_perturb": (i32, [vp, u64p, fp, i32]),
    "b2p_sign_masks": (i32, [vp, u64p, i32, C.POINTER(C.c_uint32)]),
    "b2p_mezo_eval_device": (i32, [vp, vp, vp, i32, u64p, i32, f32, vp]),
    "b2p_model_sync": (i32, [vp]),
    "b2p_model_profile": (i32, [vp, i32]),
    "b2p_model_profile_read": (i32, [vp, C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(C.c_longlong)]),
    "b2p_launch_count": (i64, []),
    "b2p_sign_masks_noalloc": (i32, [C.POINTER(C.c_int64), i32, u64p, i32, vp, vp]),
    "b2p_model_set_option": (i32, [vp, i32, i32]),
    "b2p_gemm_pair": (i32, [vp, vp, vp, i32, i32, i32, i32, i32, i32, vp]),
    "b2p_gemm_mi": (i32, [vp, vp, vp, i32, i32, i32, i32, i32, i32, vp]),
    "b2p_gemm_pair_mn": (i32, [vp, i32, i32, vp, i32, i32, vp, i32, i32, i32, i32, i32, i32, vp]),
    "b2p_p16_grad": (i32, [vp, u16p, u16p, i32, fp, vp]),
    "b2p_p16_grad_device": (i32, [vp, vp, vp, i32, vp]),
    "b2p_model_grad": (vp, [vp]),
    "b2p_adam_step": (i32, [vp, f32, f32, f32, f32, f32]),
    "b2p_adam_state": (i32, [vp, i32, ip, vp, vp]),
    "b2p_p16_step": (i32, [vp, u16p, u16p, i32, f32, fp]),
    "b2p_full_grad": (i32, [vp, u16p, u16p, i32, fp]),
    "b2p_full_update": (i32, [vp, f32, f32, f32, fp]),
    "b2p_full_step": (i32, [vp, u16p, u16p, i32, f32, f32, f32, fp, fp]),
    "b2p_full_weight_count": (i64, [vp]),
    "b2p_full_read": (i32, [vp, i32, vp, i64]),
    "b2p_ckpt_read_header": (i32, [cstr, vp]),
    "b2p_ckpt_save": (i32, [vp, cstr, cstr, vp]),
    "b2p_ckpt_load": (i32, [vp, cstr, cstr, ip, i32, i32, vp]),
    "b2p_compile": (vp, [vp, C.POINTER(fp)]),
    "b2p_input_bytes": (szt, [vp, i32]),
    "b2p_output_bytes": (szt, [vp, i32]),
    "b2p_write_input": (i32, [vp, i32, vp, szt]),
    "b2p_write_input_channels": (i32, [vp, i32, i32, i32, fp]),
    "b2p_eval": (i32, [vp]),
    "b2p_eval_async": (i32, [vp]),
    "b2p_read_output": (i32, [vp, i32, fp, szt]),
    "b2p_read_output_channels": (i32, [vp, i32, i32, i32, fp]),
    "b2p_free": (None, [vp]),
    "b2p_kernel_stream": (vp, [vp]),
    "b2p_set_lora": (i32, [vp, i32, fp, fp, i32]),
    "b2p_set_perturb": (i32, [vp, u64, f32]),
    "b2p_compile_count": (i32, []),
    "b2p_reset_compile_count": (None, []),
}


class ModelConfig(C.Structure):
    """b2p_model_config (include/b2p.h)."""
    _fields_ = [(n, C.c_int) for n in ("dim", "hidden", "heads", "kv_heads", "head_dim", "seq", "nlayers", "vocab",
                                        "rank")] + [("rope_theta", C.c_float), ("res_alpha", C.c_float),
                                                     ("dtype", C.c_int), ("max_groups", C.c_int),
                                                     ("lora_ffn", C.c_int)]


class Variant(C.Structure):
    """b2p_variant (include/b2p.h)."""
    _fields_ = [("seed", C.c_uint64), ("mode", C.c_int), ("s1", C.c_float), ("s2", C.c_float)]


class OpDesc(C.Structure):
    """b2p_op_desc (include/b2p.h)."""
    _fields_ = [(n, C.c_int) for n in ("kind", "ic", "oc", "seq", "q_dim", "kv_dim", "hidden")] + [
        ("res_alpha", C.c_float), ("dtype", C.c_int), ("n_parts", C.c_int), ("part_oc", C.c_int * 3)]


class CkptHeader(C.Structure):
    """b2p_ckpt_header: the reference's 96-byte BLZT v4 CkptHdr (training/config.h:99-108)."""
    _fields_ = [(n, C.c_int) for n in ("magic", "version", "step", "total_steps", "n_layers", "vocab_size", "dim",
                                        "hidden_dim", "n_heads", "seq_len")] + [
        ("lr", C.c_float), ("loss", C.c_float), ("cum_compile", C.c_double), ("cum_train", C.c_double),
        ("cum_wall", C.c_double)] + [(n, C.c_int) for n in ("cum_steps", "cum_batches", "adam_t", "kv_heads",
                                                              "head_dim", "q_dim")]


CKPT_MAGIC, CKPT_VERSION, LORA_MAGIC = 0x424C5A54, 4, 0x4C4F5241

OP_CONV1X1, OP_QKV_FUSED, OP_FFN_FUSED, OP_DYN_MATMUL, OP_LM_HEAD_CE, OP_DX = range(6)


class B2PError(RuntimeError):
    """A C-ABI call returned a negative status."""

    def __init__(self, name: str, rc: int, msg: str):
        super().__init__(f"{name} failed (status {rc}): {msg}")
        self.rc = rc


_lib = None


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Load libb2p.so once and bind every signature. Raises if the library is absent."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p} is missing: the CUDA library has not been built "
            "(run `python -m autoane_b200.build` or __graft_entry__.build()); there is no fallback")
    lib = C.CDLL(str(p))
    for name, (res, args) in ABI.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def call(name: str, *args):
    """Call an int-returning entry point and raise B2PError on a negative status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if isinstance(rc, int) and rc < 0:
        raise B2PError(name, rc, lib.b2p_last_error().decode(errors="replace"))
    return rc
