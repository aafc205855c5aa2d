"""Python mirror of the reference's ``DecoderLora`` (include/brosoundml/decoder_lora.h:36-164)
over the C ABI: per-AdaIN LoRA adapters on the frozen style -> (gamma, beta)
projections, the shared conditioning gate g(v) = W2 tanh(W1 v), Adam with one
shared step, and the ELRA1 checkpoint. Batched: every clip has its own style and
condition. Every computation runs in libbsml_b200.so.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .decoder import Decoder, _f32, _ptr, _stream

IN_DIM, HIDDEN = 3, 16   # ConditioningGate::in_dim, the gate hidden width (decoder_lora.cpp:141)


class DecoderLora:
    """``DecoderLora::make`` over ``decoder`` (a :class:`Decoder`); the decoder must
    outlive this object."""

    def __init__(self, decoder: Decoder, rank: int = 8, scale: float = 1.0, seed: int = 0):
        L = _lib.lib()
        h = ctypes.c_void_p()
        _lib.check(L.bsml_lora_create(decoder._h, int(rank), float(scale), int(seed), ctypes.byref(h)))
        self._h = h
        self.decoder = decoder
        n, na, r, sd = ctypes.c_int64(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        o1, o2 = ctypes.c_int64(), ctypes.c_int64()
        _lib.check(L.bsml_lora_layout(h, ctypes.byref(n), ctypes.byref(na), ctypes.byref(r), ctypes.byref(sd),
                                      ctypes.byref(o1), ctypes.byref(o2), None, None, None))
        offA = (ctypes.c_int64 * na.value)()
        offB = (ctypes.c_int64 * na.value)()
        C = (ctypes.c_int * na.value)()
        _lib.check(L.bsml_lora_layout(h, None, None, None, None, None, None, ctypes.cast(offA, ctypes.c_void_p),
                                      ctypes.cast(offB, ctypes.c_void_p), ctypes.cast(C, ctypes.c_void_p)))
        self.n_params, self.n_adapters, self.rank, self.style_dim = n.value, na.value, r.value, sd.value
        self.off_W1, self.off_W2 = o1.value, o2.value
        self.off_A, self.off_B, self.adapter_C = list(offA), list(offB), list(C)
        pp, gp = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(L.bsml_lora_buffers(h, ctypes.byref(pp), ctypes.byref(gp)))
        self._pp, self._gp = pp.value, gp.value

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and _lib._lib is not None:
            _lib.lib().bsml_lora_destroy(h)
            self._h = None

    # ── the flat parameter / gradient vectors, as torch views of the object's device memory
    def params(self) -> torch.Tensor:
        """View (no copy) of the flat parameter vector: gate W1 [16][3], gate W2 [rank][16],
        then per adapter A [rank][style_dim] (at off_A[a]) and B [2C][rank] (at off_B[a])."""
        return _device_view(self._pp, self.n_params, self.decoder.device)

    def grads(self) -> torch.Tensor:
        """View (no copy) of the flat gradient vector (same layout as :meth:`params`)."""
        return _device_view(self._gp, self.n_params, self.decoder.device)

    @property
    def scale(self) -> float:
        s, st = ctypes.c_float(), ctypes.c_int()
        _lib.check(_lib.lib().bsml_lora_state(self._h, ctypes.byref(s), ctypes.byref(st)))
        return s.value

    @property
    def step(self) -> int:
        s, st = ctypes.c_float(), ctypes.c_int()
        _lib.check(_lib.lib().bsml_lora_state(self._h, ctypes.byref(s), ctypes.byref(st)))
        return st.value

    # ── DecoderLora::forward / backward / zero_grad / adam_step / save / load
    def forward(self, params, asr, F0, N, ref_s, cond, har=None, audio=None):
        params, asr, F0, N, ref_s, cond, har = map(_f32, (params, asr, F0, N, ref_s, cond, har))
        B, _, T = asr.shape
        frames = 0 if har is None else har.shape[2]
        if audio is None:
            audio = torch.empty((B, self.decoder.audio_len(T, frames if har is not None else None)),
                                device=self.decoder.device)
        self._borrowed = params   # the engine reads the weights again in the backward
        _lib.check(_lib.lib().bsml_lora_forward(self._h, B, T, _ptr(params), _ptr(asr), _ptr(F0), _ptr(N),
                                                _ptr(ref_s), ref_s.shape[-1], _ptr(har), frames, _ptr(cond),
                                                _ptr(audio), _stream()))
        return audio

    def backward(self, daudio) -> None:
        _lib.check(_lib.lib().bsml_lora_backward(self._h, _ptr(_f32(daudio)), _stream()))

    def zero_grad(self) -> None:
        _lib.check(_lib.lib().bsml_lora_zero_grad(self._h, _stream()))

    def adam_step(self, lr: float, beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8) -> None:
        _lib.check(_lib.lib().bsml_lora_adam_step(self._h, lr, beta1, beta2, eps, _stream()))

    def save(self, path: str, full_state: bool = False) -> None:
        """ELRA1 checkpoint; full_state adds Adam's moments and step after it (the
        file stays readable by the plain-format readers)."""
        fn = _lib.lib().bsml_lora_save_state if full_state else _lib.lib().bsml_lora_save
        _lib.check(fn(self._h, str(path).encode()))

    def load(self, path: str, full_state: bool = False) -> None:
        fn = _lib.lib().bsml_lora_load_state if full_state else _lib.lib().bsml_lora_load
        _lib.check(fn(self._h, str(path).encode()))


class _DeviceBuffer:
    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}


def _device_view(ptr: int, n: int, device) -> torch.Tensor:
    return torch.as_tensor(_DeviceBuffer(ptr, n), device=device)


class ConvLora:
    """Conv-weight LoRA (the fine-tune of every conv weight; no counterpart in the reference): a rank-r
    adapter W + scale * B A on every Conv1d / ConvTranspose1d weight of ``decoder``,
    base weights frozen. A weight stored (d0, d1, k) is viewed as [d0][d1*k];
    A [rank][d1*k] starts N(0, 0.01), B [d0][rank] starts at zero."""

    def __init__(self, decoder: Decoder, rank: int = 8, scale: float = 2.0, seed: int = 0):
        L = _lib.lib()
        h = ctypes.c_void_p()
        _lib.check(L.bsml_convlora_create(decoder._h, int(rank), float(scale), int(seed), ctypes.byref(h)))
        self._h, self.decoder, self.rank, self.scale = h, decoder, int(rank), float(scale)
        n, nw = ctypes.c_int64(), ctypes.c_int()
        _lib.check(L.bsml_convlora_layout(h, ctypes.byref(n), ctypes.byref(nw), None, None, None, None, None))
        arrs = [(ctypes.c_int64 * nw.value)(), (ctypes.c_int * nw.value)(), (ctypes.c_int * nw.value)(),
                (ctypes.c_int64 * nw.value)(), (ctypes.c_int64 * nw.value)()]
        _lib.check(L.bsml_convlora_layout(h, None, None, *[ctypes.cast(a, ctypes.c_void_p) for a in arrs]))
        self.n_params = n.value
        self.weights = [dict(w=w, rows=r, cols=c, offA=a, offB=b) for w, r, c, a, b in zip(*[list(a) for a in arrs])]
        pp, gp = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(L.bsml_convlora_buffers(h, ctypes.byref(pp), ctypes.byref(gp)))
        self._pp, self._gp = pp.value, gp.value

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and _lib._lib is not None:
            _lib.lib().bsml_convlora_destroy(h)
            self._h = None

    def params(self) -> torch.Tensor:
        return _device_view(self._pp, self.n_params, self.decoder.device)

    def grads(self) -> torch.Tensor:
        return _device_view(self._gp, self.n_params, self.decoder.device)

    def forward(self, params, asr, F0, N, style, har=None, audio=None):
        params, asr, F0, N, style, har = map(_f32, (params, asr, F0, N, style, har))
        B, _, T = asr.shape
        frames = 0 if har is None else har.shape[2]
        if audio is None:
            audio = torch.empty((B, self.decoder.audio_len(T, frames if har is not None else None)),
                                device=self.decoder.device)
        _lib.check(_lib.lib().bsml_convlora_forward(self._h, B, T, _ptr(params), _ptr(asr), _ptr(F0), _ptr(N),
                                                    _ptr(style), _ptr(har), frames, _ptr(audio), _stream()))
        return audio

    def backward(self, daudio) -> None:
        _lib.check(_lib.lib().bsml_convlora_backward(self._h, _ptr(_f32(daudio)), _stream()))

    def zero_grad(self) -> None:
        _lib.check(_lib.lib().bsml_convlora_zero_grad(self._h, _stream()))

    def adam_step(self, lr: float, beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8) -> None:
        _lib.check(_lib.lib().bsml_convlora_adam_step(self._h, lr, beta1, beta2, eps, _stream()))

    def save(self, path: str) -> None:
        """Full training state (ECLR1): A, B, Adam moments and step."""
        _lib.check(_lib.lib().bsml_convlora_save(self._h, str(path).encode()))

    def load(self, path: str) -> None:
        _lib.check(_lib.lib().bsml_convlora_load(self._h, str(path).encode()))
