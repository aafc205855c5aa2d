"""ctypes wrapper over the CPU oracle (libkokoro_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
the CPU-baseline leg of ``bench.py``; never by the product package.

PARITY STATUS: unpinned by reference artefacts (the reference's arithmetic lives
in the absent ``brotensor`` library and no golden vectors exist for this path).
Pinned instead by oracle/torch_decoder.py (independent autograd restatement)
and by the reference's finite-difference methodology, run in float64.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libkokoro_oracle.so")


class OrcCfg(ctypes.Structure):
    """Mirror of ``orc_cfg`` in kokoro_oracle.cpp (architecture description)."""

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


class OrcParam(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 96), ("offset", ctypes.c_int64), ("numel", ctypes.c_int64),
                ("ndim", ctypes.c_int), ("shape", ctypes.c_int * 3), ("trainable", ctypes.c_int)]


class OrcBlockSpec(ctypes.Structure):
    """Mirror of ``orc_block_spec``: kind 1 = AdainResBlk1d, kind 2 = AdaINResBlock1."""

    _fields_ = [("kind", ctypes.c_int), ("style_dim", ctypes.c_int), ("cin", ctypes.c_int), ("cout", ctypes.c_int),
                ("upsample", ctypes.c_int), ("kernel", ctypes.c_int), ("dil", ctypes.c_int * 3)]


def make_block_spec(d: dict) -> OrcBlockSpec:
    s = OrcBlockSpec()
    for k, v in d.items():
        if k == "dil":
            for i, x in enumerate(v):
                s.dil[i] = int(x)
        else:
            setattr(s, k, int(v))
    return s


def make_cfg(d: dict) -> OrcCfg:
    """Build an OrcCfg from a plain dict (the same dict the product accepts)."""
    c = OrcCfg()
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


def build(force: bool = False) -> str:
    if force or not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "kokoro_oracle.cpp"))):
        subprocess.run(["make", "-C", _HERE], check=True, capture_output=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        I = ctypes.c_int
        _lib.orc_param_count.argtypes = [ctypes.POINTER(OrcCfg), ctypes.POINTER(ctypes.c_int64),
                                         ctypes.POINTER(I), ctypes.POINTER(I), ctypes.POINTER(ctypes.c_int64)]
        _lib.orc_param_table.argtypes = [ctypes.POINTER(OrcCfg), ctypes.POINTER(OrcParam), I, P]
        for sfx in ("f32", "f64"):
            fn = getattr(_lib, f"orc_decoder_run_{sfx}")
            fn.argtypes = [ctypes.POINTER(OrcCfg), I, I] + [P] * 6 + [I] + [P] * 8
        BS = ctypes.POINTER(OrcBlockSpec)
        _lib.orc_block_param_count.argtypes = [BS, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(I),
                                               ctypes.POINTER(I), ctypes.POINTER(ctypes.c_int64)]
        _lib.orc_block_param_table.argtypes = [BS, ctypes.POINTER(OrcParam), I, P]
        for sfx in ("f32", "f64"):
            getattr(_lib, f"orc_block_run_{sfx}").argtypes = [BS, I, I] + [P] * 11
        _lib.orc_harmonic_source_f32.argtypes = [ctypes.POINTER(OrcCfg), P, I, I, P, P, P]
        _lib.orc_threads.restype = I
        _lib.orc_set_threads.argtypes = [I]
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


class BlockOracle:
    """One decoder block on its own: ``spec`` = dict(kind=1, style_dim, cin, cout, upsample)
    for an AdainResBlk1d or dict(kind=2, style_dim, cin=C, cout=C, kernel, dil) for an
    AdaINResBlock1 (src/kokoro_decoder_backward.h:82-144)."""

    def __init__(self, spec: dict):
        self.spec_dict = dict(spec)
        self.spec = make_block_spec(spec)
        L = lib()
        tot, ne, na, apc = ctypes.c_int64(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int64()
        L.orc_block_param_count(ctypes.byref(self.spec), ctypes.byref(tot), ctypes.byref(ne), ctypes.byref(na),
                                ctypes.byref(apc))
        self.n_params, self.n_affine, self.aff_per_clip = tot.value, na.value, apc.value
        arr = (OrcParam * ne.value)()
        affc = np.zeros(na.value, dtype=np.int32)
        L.orc_block_param_table(ctypes.byref(self.spec), arr, ne.value, _p(affc))
        self.table = [dict(name=p.name.decode(), offset=p.offset, numel=p.numel,
                           shape=tuple(p.shape[:p.ndim]), trainable=bool(p.trainable)) for p in arr]
        self.aff_C = [int(c) for c in affc]

    def out_len(self, L: int) -> int:
        return 2 * L if self.spec_dict["kind"] == 1 and self.spec_dict.get("upsample") else L

    def run(self, params, x, style, aff_in=None, dy=None, dtype=np.float32, want_aff=False):
        """x (B, cin, L) NCL; style (B, style_dim); aff_in packed (gamma, beta) or None; dy
        (B, cout, L_out) for the backward. Returns y and, with dy, grads, dx, d_style, d_aff."""
        B, _, L = x.shape
        f = (lambda a: None if a is None else np.ascontiguousarray(a, dtype=dtype))
        params, x, style, aff_in, dy = map(f, (params, x, style, aff_in, dy))
        out = dict(y=np.zeros((B, self.spec_dict["cout"], self.out_len(L)), dtype))
        if dy is not None:
            out["grads"] = np.zeros(self.n_params, dtype)
            out["dx"] = np.zeros_like(x)
            out["d_style"] = np.zeros((B, self.spec_dict["style_dim"]), dtype)
            out["d_aff"] = np.zeros(B * self.aff_per_clip, dtype)
        if want_aff:
            out["aff"] = np.zeros(B * self.aff_per_clip, dtype)
        fn = lib().orc_block_run_f32 if dtype == np.float32 else lib().orc_block_run_f64
        rc = fn(ctypes.byref(self.spec), B, L, _p(params), _p(x), _p(style), _p(aff_in), _p(dy), _p(out["y"]),
                _p(out.get("grads")), _p(out.get("dx")), _p(out.get("d_style")), _p(out.get("d_aff")),
                _p(out.get("aff")))
        if rc != 0:
            raise RuntimeError(f"oracle: block run failed ({rc})")
        return out


class Oracle:
    """The oracle for one architecture ``cfg`` (a dict, see brosoundml_b200.config)."""

    def __init__(self, cfg: dict):
        self.cfg_dict = dict(cfg)
        self.cfg = make_cfg(cfg)
        L = lib()
        tot, ne, na, apc = ctypes.c_int64(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int64()
        L.orc_param_count(ctypes.byref(self.cfg), ctypes.byref(tot), ctypes.byref(ne), ctypes.byref(na),
                          ctypes.byref(apc))
        self.n_params = tot.value
        self.n_affine = na.value
        self.aff_per_clip = apc.value
        arr = (OrcParam * ne.value)()
        affc = np.zeros(na.value, dtype=np.int32)
        L.orc_param_table(ctypes.byref(self.cfg), arr, ne.value, _p(affc))
        self.table = [dict(name=p.name.decode(), offset=p.offset, numel=p.numel,
                           shape=tuple(p.shape[:p.ndim]), trainable=bool(p.trainable)) for p in arr]
        self.aff_C = [int(c) for c in affc]

    def run(self, params, asr, F0, N, style, har=None, aff_in=None, daudio=None, dtype=np.float32,
            want_aff=False):
        """Forward (and backward when ``daudio`` is given) of the whole decoder.

        Shapes: asr (B, asr_dim, T); F0/N (B, 2T); style (B, style_dim);
        har (B, har_ch, frames) or None to run the harmonic source; aff_in:
        (B * aff_per_clip,) packed per-AdaIN (gamma, beta) blocks (reference mode)
        or None to use fc(style). Returns a dict of numpy arrays.
        """
        c = self.cfg_dict
        B, _, T = asr.shape
        if har is None and c["har_ch"] != c["n_fft"] + 2:
            raise ValueError("oracle: the harmonic source makes n_fft + 2 channels; "
                             f"this config has har_ch = {c['har_ch']}: pass har")
        f = (lambda a: None if a is None else np.ascontiguousarray(a, dtype=dtype))
        params, asr, F0, N, style, har, aff_in, daudio = map(f, (params, asr, F0, N, style, har, aff_in, daudio))
        L_last_frames = (2 * T * c["upsample_scale"]) // c["hop"] + 1 if har is None else har.shape[2]
        S = c["hop"] * (L_last_frames - 1)
        out = dict(audio=np.zeros((B, S), dtype))
        if daudio is not None:
            out["grads"] = np.zeros(self.n_params, dtype)
            out["d_asr"] = np.zeros_like(asr)
            out["d_style"] = np.zeros_like(style)
            out["d_aff"] = np.zeros(B * self.aff_per_clip, dtype)
        if want_aff:
            out["aff"] = np.zeros(B * self.aff_per_clip, dtype)
        fn = lib().orc_decoder_run_f32 if dtype == np.float32 else lib().orc_decoder_run_f64
        rc = fn(ctypes.byref(self.cfg), B, T, _p(params), _p(asr), _p(F0), _p(N), _p(style), _p(har),
                0 if har is None else har.shape[2], _p(aff_in), _p(daudio), _p(out["audio"]),
                _p(out.get("grads")), _p(out.get("d_asr")), _p(out.get("d_style")), _p(out.get("d_aff")),
                _p(out.get("aff")))
        if rc != 0:
            raise RuntimeError(f"oracle: decoder run failed ({rc})")
        return out

    def harmonic_source(self, params, F0):
        c = self.cfg_dict
        B, Fr = F0.shape
        frames = (Fr * c["upsample_scale"]) // c["hop"] + 1
        har = np.zeros((B, c["har_ch"], frames), np.float32)
        lw = next(p for p in self.table if p["name"] == "generator.m_source.l_linear.weight")
        lb = next(p for p in self.table if p["name"] == "generator.m_source.l_linear.bias")
        params = np.ascontiguousarray(params, np.float32)
        F0 = np.ascontiguousarray(F0, np.float32)
        lib().orc_harmonic_source_f32(ctypes.byref(self.cfg), _p(F0), B, Fr,
                                      _p(params[lw["offset"]:]), _p(params[lb["offset"]:]), _p(har))
        return har

    # ── atom-level ops (float32 or float64 by array dtype)
    def _atom(self, name, dtype):
        fn = getattr(lib(), f"orc_{name}_{'f32' if dtype == np.float32 else 'f64'}")
        return fn

    def conv_fwd(self, x, W, b, stride, pad, dil):
        B, Ci, L = x.shape
        Co, _, k = W.shape
        Lo = (L + 2 * pad - dil * (k - 1) - 1) // stride + 1
        y = np.zeros((B, Co, Lo), x.dtype)
        fn = self._atom("conv_fwd", x.dtype)
        I = ctypes.c_int
        fn(_p(x), I(B), I(Ci), I(L), _p(W), _p(b), I(Co), I(k), I(stride), I(pad), I(dil), _p(y))
        return y

    def conv_dgrad(self, dy, W, L, stride, pad, dil):
        B, Co, _ = dy.shape
        _, Ci, k = W.shape
        dx = np.zeros((B, Ci, L), dy.dtype)
        I = ctypes.c_int
        self._atom("conv_dgrad", dy.dtype)(_p(dy), I(B), I(Ci), I(L), _p(W), I(Co), I(k), I(stride), I(pad),
                                           I(dil), _p(dx))
        return dx

    def conv_wgrad(self, dy, x, k, stride, pad, dil):
        B, Co, _ = dy.shape
        _, Ci, L = x.shape
        dW = np.zeros((Co, Ci, k), dy.dtype)
        db = np.zeros(Co, dy.dtype)
        I = ctypes.c_int
        self._atom("conv_wgrad", dy.dtype)(_p(dy), _p(x), I(B), I(Ci), I(L), I(Co), I(k), I(stride), I(pad),
                                           I(dil), _p(dW), _p(db))
        return dW, db

    def convT_fwd(self, x, W, b, stride, pad):
        B, Ci, L = x.shape
        _, Co, k = W.shape
        Lo = (L - 1) * stride - 2 * pad + k
        y = np.zeros((B, Co, Lo), x.dtype)
        I = ctypes.c_int
        self._atom("convT_fwd", x.dtype)(_p(x), I(B), I(Ci), I(L), _p(W), _p(b), I(Co), I(k), I(stride), I(pad),
                                         _p(y))
        return y

    def convT_dgrad(self, dy, W, L, stride, pad):
        B, Co, _ = dy.shape
        Ci, _, k = W.shape
        dx = np.zeros((B, Ci, L), dy.dtype)
        I = ctypes.c_int
        self._atom("convT_dgrad", dy.dtype)(_p(dy), I(B), I(Ci), I(L), _p(W), I(Co), I(k), I(stride), I(pad),
                                           _p(dx))
        return dx

    def convT_wgrad(self, dy, x, k, stride, pad):
        B, Co, _ = dy.shape
        _, Ci, L = x.shape
        dW = np.zeros((Ci, Co, k), dy.dtype)
        db = np.zeros(Co, dy.dtype)
        I = ctypes.c_int
        self._atom("convT_wgrad", dy.dtype)(_p(dy), _p(x), I(B), I(Ci), I(L), I(Co), I(k), I(stride), I(pad),
                                           _p(dW), _p(db))
        return dW, db

    def adain_fwd(self, x, gb, eps=1e-5):
        B, C, L = x.shape
        y = np.zeros_like(x)
        I = ctypes.c_int
        R = ctypes.c_float if x.dtype == np.float32 else ctypes.c_double
        self._atom("adain_fwd", x.dtype)(_p(x), I(B), I(C), I(L), _p(gb), R(eps), _p(y))
        return y

    def adain_bwd(self, x, gb, dy, eps=1e-5):
        B, C, L = x.shape
        dx = np.zeros_like(x)
        dgb = np.zeros_like(gb)
        I = ctypes.c_int
        R = ctypes.c_float if x.dtype == np.float32 else ctypes.c_double
        self._atom("adain_bwd", x.dtype)(_p(x), I(B), I(C), I(L), _p(gb), R(eps), _p(dy), _p(dx), _p(dgb))
        return dx, dgb

    def snake_fwd(self, x, alpha):
        B, C, L = x.shape
        y = np.zeros_like(x)
        I = ctypes.c_int
        self._atom("snake_fwd", x.dtype)(_p(x), I(B), I(C), I(L), _p(alpha), _p(y))
        return y

    def snake_bwd(self, x, alpha, dy):
        B, C, L = x.shape
        dx = np.zeros_like(x)
        da = np.zeros_like(alpha)
        I = ctypes.c_int
        self._atom("snake_bwd", x.dtype)(_p(x), I(B), I(C), I(L), _p(alpha), _p(dy), _p(dx), _p(da))
        return dx, da

    def istft_fwd(self, re, im, n_fft, hop):
        B, nf, L = re.shape
        a = np.zeros((B, hop * (L - 1)), re.dtype)
        I = ctypes.c_int
        self._atom("istft_fwd", re.dtype)(_p(re), _p(im), I(B), I(n_fft), I(hop), I(L), _p(a))
        return a

    def istft_bwd(self, da, n_fft, hop, L):
        B = da.shape[0]
        nf = n_fft // 2 + 1
        dre = np.zeros((B, nf, L), da.dtype)
        dim = np.zeros((B, nf, L), da.dtype)
        I = ctypes.c_int
        self._atom("istft_bwd", da.dtype)(_p(da), I(B), I(n_fft), I(hop), I(L), _p(dre), _p(dim))
        return dre, dim


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def threads() -> int:
    return int(lib().orc_threads())
