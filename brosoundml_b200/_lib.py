"""ctypes binding of libbsml_b200.so (include/bsml_decoder.h).

The product path has no fallback: if the CUDA library is missing this module
raises, it never substitutes a CPU implementation.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# BSML_LIB selects another build of the library (e.g. the DEBUG=1 bounds-checking one)
LIB_PATH = os.environ.get("BSML_LIB") or os.path.join(_HERE, "libbsml_b200.so")


class BsmlConfig(ctypes.Structure):
    """Mirror of bsml_decoder_config."""

    _fields_ = [
        ("asr_dim", ctypes.c_int), ("style_dim", ctypes.c_int), ("asr_res_dim", ctypes.c_int),
        ("enc_dim", ctypes.c_int), ("n_decode", ctypes.c_int), ("dec_out", ctypes.c_int * 8),
        ("upsample_block", ctypes.c_int), ("n_ups", ctypes.c_int), ("init_ch", ctypes.c_int),
        ("ups_rate", ctypes.c_int * 4), ("ups_kernel", ctypes.c_int * 4),
        ("noise_kernel", ctypes.c_int * 4), ("noise_stride", ctypes.c_int * 4),
        ("noise_pad", ctypes.c_int * 4), ("nr_kernel", ctypes.c_int * 4),
        ("nr_dil", (ctypes.c_int * 3) * 4), ("n_kernels", ctypes.c_int),
        ("rb_kernel", ctypes.c_int * 4), ("rb_dil", (ctypes.c_int * 3) * 4),
        ("har_ch", ctypes.c_int), ("n_fft", ctypes.c_int), ("hop", ctypes.c_int),
        ("post_kernel", ctypes.c_int), ("harmonic_num", ctypes.c_int),
        ("sample_rate", ctypes.c_int), ("upsample_scale", ctypes.c_int),
    ]


class BsmlParamEntry(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 96), ("offset", ctypes.c_int64), ("numel", ctypes.c_int64),
                ("ndim", ctypes.c_int), ("shape", ctypes.c_int * 3), ("trainable", ctypes.c_int)]


class BsmlBlockSpec(ctypes.Structure):
    """Mirror of bsml_block_spec (kind 1 = AdainResBlk1d, 2 = AdaINResBlock1)."""

    _fields_ = [("kind", ctypes.c_int), ("style_dim", ctypes.c_int), ("cin", ctypes.c_int), ("cout", ctypes.c_int),
                ("upsample", ctypes.c_int), ("kernel", ctypes.c_int), ("dil", ctypes.c_int * 3)]


def make_block_spec(d: dict) -> BsmlBlockSpec:
    s = BsmlBlockSpec()
    for k, v in d.items():
        if k == "dil":
            for i, x in enumerate(v):
                s.dil[i] = int(x)
        else:
            setattr(s, k, int(v))
    return s


def make_config(d: dict) -> BsmlConfig:
    c = BsmlConfig()
    for k, v in d.items():
        f = getattr(c, k)
        if isinstance(v, (list, tuple)):
            if v and isinstance(v[0], (list, tuple)):
                for i, row in enumerate(v):
                    for j, x in enumerate(row):
                        f[i][j] = int(x)
            else:
                for i, x in enumerate(v):
                    f[i] = int(x)
        else:
            setattr(c, k, int(v))
    return c


# Every exported entry point with its argument types (restype int unless noted).
_P, _I, _F, _L = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_int64
_CFG = ctypes.POINTER(BsmlConfig)
_BS = ctypes.POINTER(BsmlBlockSpec)
SIGNATURES = {
    "bsml_last_error": ([], ctypes.c_char_p),
    "bsml_version": ([], _I),
    "bsml_decoder_create": ([_CFG, _I, ctypes.POINTER(_P)], _I),
    "bsml_decoder_destroy": ([_P], None),
    "bsml_decoder_param_count": ([_P, ctypes.POINTER(_L), ctypes.POINTER(_I), ctypes.POINTER(_I),
                                  ctypes.POINTER(_L)], _I),
    "bsml_decoder_param_table": ([_P, _P, _I, _P], _I),
    "bsml_decoder_set_math": ([_P, _I], _I),
    "bsml_config_param_count": ([_CFG, ctypes.POINTER(_L), ctypes.POINTER(_I), ctypes.POINTER(_I),
                                 ctypes.POINTER(_L)], _I),
    "bsml_config_param_table": ([_CFG, _P, _I, _P], _I),
    "bsml_decoder_forward": ([_P, _I, _I, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P], _I),
    "bsml_decoder_backward": ([_P, _P, _P, _P, _P, _P, _P], _I),
    "bsml_decoder_decode": ([_P, _I, _I, _P, _P, _I, _P, _P, _P, _P, _P], _I),
    "bsml_decoder_workspace_bytes": ([_P], _L),
    "bsml_selftest_bounded_wait": ([_P], _I),
    "bsml_st_open": ([ctypes.c_char_p, ctypes.POINTER(_P)], _I),
    "bsml_st_close": ([_P], None),
    "bsml_st_count": ([_P, ctypes.POINTER(_I)], _I),
    "bsml_st_info": ([_P, _I, ctypes.c_char_p, _I, ctypes.POINTER(_I), ctypes.POINTER(_I), _P], _I),
    "bsml_st_read_f32": ([_P, ctypes.c_char_p, _P, _L], _I),
    "bsml_st_metadata": ([_P, ctypes.c_char_p, ctypes.c_char_p, _I], _I),
    "bsml_params_from_safetensors": ([_P, _P, _I, ctypes.c_char_p, _P, _L], _I),
    "bsml_nccl_unique_id": ([_P], _I),
    "bsml_nccl_version": ([ctypes.POINTER(_I)], _I),
    "bsml_nccl_comm_init": ([_I, _P, _I, _I, ctypes.POINTER(_P)], _I),
    "bsml_nccl_comm_init_timeout": ([_I, _P, _I, _I, _I, ctypes.POINTER(_P)], _I),
    "bsml_nccl_comm_destroy": ([_P], _I),
    "bsml_allreduce_grads": ([_P, _P, _L, _I, _P], _I),
    "bsml_nccl_sync": ([_P, _P], _I),
    "bsml_graph_begin": ([_P], _I),
    "bsml_graph_end": ([_P, ctypes.POINTER(_P)], _I),
    "bsml_graph_launch": ([_P, _P], _I),
    "bsml_graph_kernel_count": ([_P, ctypes.POINTER(_L)], _I),
    "bsml_graph_destroy": ([_P], None),
    "bsml_block_create": ([_BS, _I, ctypes.POINTER(_P)], _I),
    "bsml_block_param_count": ([_BS, ctypes.POINTER(_L), ctypes.POINTER(_I), ctypes.POINTER(_I),
                                ctypes.POINTER(_L)], _I),
    "bsml_block_param_table": ([_BS, _P, _I, _P], _I),
    "bsml_block_forward": ([_P, _I, _I, _P, _P, _P, _P, _P, _P, _P], _I),
    "bsml_block_backward": ([_P, _P, _P, _P, _P, _P, _P], _I),
    "bsml_decoder_set_profiling": ([_P, _I], _I),
    "bsml_launch_count": ([], _L),
    "bsml_set_atom_math": ([_I], _I),
    "bsml_device_error": ([], _I),
    "bsml_decoder_read_profile": ([_P, _P], _I),
    "bsml_decoder_read_profile_records": ([_P, _P, _I, _P], _I),
    "bsml_loss_l1": ([_P, _P, _L, _P, _P, _P], _I),
    "bsml_adam_step": ([_P, _P, _P, _P, _L, _F, _F, _F, _F, _I, _P], _I),
    "bsml_conv1d_forward": ([_P, _I, _I, _I, _P, _P, _I, _I, _I, _I, _I, _P, _P], _I),
    "bsml_conv1d_backward_input": ([_P, _I, _I, _I, _P, _I, _I, _I, _I, _I, _P, _P], _I),
    "bsml_conv1d_backward_weight": ([_P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P], _I),
    "bsml_conv1d_backward_weight_noalloc": ([_P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P], _I),
    "bsml_conv_transpose1d_forward": ([_P, _I, _I, _I, _P, _P, _I, _I, _I, _I, _P, _P], _I),
    "bsml_conv_transpose1d_backward_input": ([_P, _I, _I, _I, _P, _I, _I, _I, _I, _P, _P], _I),
    "bsml_conv_transpose1d_backward_weight": ([_P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P], _I),
    "bsml_adain_affine_forward": ([_P, _P, _I, _I, _I, _F, _P, _P], _I),
    "bsml_adain_affine_backward": ([_P, _P, _P, _I, _I, _I, _F, _P, _P, _P], _I),
    "bsml_snake_forward": ([_P, _P, _I, _I, _I, _P, _P], _I),
    "bsml_snake_backward": ([_P, _P, _P, _I, _I, _I, _P, _P, _P], _I),
    "bsml_istft_forward": ([_P, _P, _I, _I, _I, _I, _P, _P], _I),
    "bsml_istft_backward": ([_P, _I, _I, _I, _I, _P, _P, _P], _I),
    "bsml_backbone_out_len": ([_P, _I, ctypes.POINTER(_I)], _I),
    "bsml_backbone_forward": ([_P, _I, _I, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P], _I),
    "bsml_backbone_backward": ([_P, _P, _P, _P, _P, _P, _P], _I),
    "bsml_generator_forward": ([_P, _I, _I, _P, _P, _P, _I, _P, _I, _P, _P, _P, _P], _I),
    "bsml_generator_backward": ([_P, _P, _P, _P, _P, _P, _P], _I),
    "bsml_spectral_head_forward": ([_P, _I, _I, _I, _P, _P, _I, _I, _I, _P, _P, _P], _I),
    "bsml_spectral_head_backward": ([_P, _P, _P, _I, _I, _I, _P, _I, _I, _I, _P, _P], _I),
    "bsml_transpose": ([_P, _L, _I, _I, _P, _P], _I),
    "bsml_managed_alloc": ([_L, ctypes.POINTER(_P)], _I),
    "bsml_managed_free": ([_P], _I),
    "bsml_synchronize": ([], _I),
    "bsml_memcpy": ([_P, _P, _L, _P], _I),
    "bsml_lora_moments": ([_P, ctypes.POINTER(_P), ctypes.POINTER(_P)], _I),
    "bsml_gate_forward": ([_P, _P, _P, _I, _I, _I, _I, _P, _P, _P], _I),
    "bsml_gate_backward": ([_P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P], _I),
    "bsml_debug_bounds": ([_P], _I),
    "bsml_harmonic_source": ([_CFG, _P, _I, _I, _P, _P, _P, _P], _I),
    "bsml_harmonic_source_mode": ([_CFG, _P, _I, _I, _P, _P, _P, _I, _P], _I),
    "bsml_decoder_set_phase_mode": ([_P, _I], _I),
    "bsml_lora_create": ([_P, _I, _F, ctypes.c_uint64, ctypes.POINTER(_P)], _I),
    "bsml_lora_destroy": ([_P], None),
    "bsml_lora_layout": ([_P, ctypes.POINTER(_L), ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I),
                          ctypes.POINTER(_L), ctypes.POINTER(_L), _P, _P, _P], _I),
    "bsml_lora_buffers": ([_P, ctypes.POINTER(_P), ctypes.POINTER(_P)], _I),
    "bsml_lora_forward": ([_P, _I, _I, _P, _P, _P, _P, _P, _I, _P, _I, _P, _P, _P], _I),
    "bsml_lora_backward": ([_P, _P, _P], _I),
    "bsml_lora_zero_grad": ([_P, _P], _I),
    "bsml_lora_adam_step": ([_P, _F, _F, _F, _F, _P], _I),
    "bsml_lora_save": ([_P, ctypes.c_char_p], _I),
    "bsml_lora_load": ([_P, ctypes.c_char_p], _I),
    "bsml_lora_state": ([_P, ctypes.POINTER(_F), ctypes.POINTER(_I)], _I),
    "bsml_convlora_create": ([_P, _I, _F, ctypes.c_uint64, ctypes.POINTER(_P)], _I),
    "bsml_convlora_destroy": ([_P], None),
    "bsml_convlora_layout": ([_P, ctypes.POINTER(_L), ctypes.POINTER(_I), _P, _P, _P, _P, _P], _I),
    "bsml_convlora_buffers": ([_P, ctypes.POINTER(_P), ctypes.POINTER(_P)], _I),
    "bsml_convlora_forward": ([_P, _I, _I, _P, _P, _P, _P, _P, _P, _I, _P, _P], _I),
    "bsml_convlora_backward": ([_P, _P, _P], _I),
    "bsml_convlora_zero_grad": ([_P, _P], _I),
    "bsml_convlora_adam_step": ([_P, _F, _F, _F, _F, _P], _I),
    "bsml_convlora_save": ([_P, ctypes.c_char_p], _I),
    "bsml_convlora_load": ([_P, ctypes.c_char_p], _I),
    "bsml_lora_save_state": ([_P, ctypes.c_char_p], _I),
    "bsml_lora_load_state": ([_P, ctypes.c_char_p], _I),
}

_lib = None


class BsmlError(RuntimeError):
    pass


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise BsmlError(f"brosoundml: CUDA library not built ({LIB_PATH}); run __graft_entry__.build()")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != 0:
        raise BsmlError(lib().bsml_last_error().decode())


def block_layout(spec: dict):
    """Parameter table of one block without a device: (n_params, table, aff_C, aff_per_clip)."""
    L = lib()
    c = make_block_spec(spec)
    n, ne, na, apc = ctypes.c_int64(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int64()
    check(L.bsml_block_param_count(ctypes.byref(c), ctypes.byref(n), ctypes.byref(ne), ctypes.byref(na),
                                   ctypes.byref(apc)))
    arr = (BsmlParamEntry * ne.value)()
    affc = (ctypes.c_int * na.value)()
    rc = L.bsml_block_param_table(ctypes.byref(c), ctypes.cast(arr, ctypes.c_void_p), ne.value,
                                  ctypes.cast(affc, ctypes.c_void_p))
    if rc < 0:
        check(rc)
    table = [dict(name=e.name.decode(), offset=e.offset, numel=e.numel, shape=tuple(e.shape[:e.ndim]),
                  trainable=bool(e.trainable)) for e in arr]
    return n.value, table, list(affc), apc.value


def layout(cfg: dict):
    """Parameter table of a config without a device: (n_params, table, aff_C, aff_per_clip)."""
    L = lib()
    c = make_config(cfg)
    n, ne, na, apc = ctypes.c_int64(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int64()
    check(L.bsml_config_param_count(ctypes.byref(c), ctypes.byref(n), ctypes.byref(ne), ctypes.byref(na),
                                    ctypes.byref(apc)))
    arr = (BsmlParamEntry * ne.value)()
    affc = (ctypes.c_int * na.value)()
    rc = L.bsml_config_param_table(ctypes.byref(c), ctypes.cast(arr, ctypes.c_void_p), ne.value,
                                   ctypes.cast(affc, ctypes.c_void_p))
    if rc < 0:
        check(rc)
    table = [dict(name=e.name.decode(), offset=e.offset, numel=e.numel, shape=tuple(e.shape[:e.ndim]),
                  trainable=bool(e.trainable)) for e in arr]
    return n.value, table, list(affc), apc.value
