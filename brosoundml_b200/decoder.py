"""Python host mirror of the reference's decoder training interface, over the C ABI.

``Decoder`` wraps one ``bsml_decoder`` engine (forward with caches, backward),
``DecoderLora``-style training loops are built from it in ``train.py``.
Tensors are torch CUDA tensors (torch is the device-memory and stream
plumbing here; every computation runs in libbsml_b200.so).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

MATH = {"fp32": 0, "tf32x3": 1, "bf16": 2, "bf16x3": 3, "tf32x3w": 4, "tf32x3f": 5}
PHASE = {"fp32": 0, "exact": 1}


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _f32(t):
    if t is None:
        return None
    if not (t.is_cuda and t.dtype == torch.float32):
        raise TypeError("brosoundml: expected a float32 CUDA tensor")
    return t.contiguous()


class Decoder:
    # math modes smoke() exercises (the tensor-core modes join once built)
    SMOKE_MATH = ("fp32", "tf32x3", "bf16x3")
    # the fp32-grade tensor-core mode (bench.py runs "tf32x3f": TF32x3 forward, BF16x3
    # backward, within the same bar at config 2)
    DEFAULT_MATH = "tf32x3"

    def __init__(self, cfg: dict, device: int = 0, math: str = "fp32"):
        self.cfg = dict(cfg)
        self._c = _lib.make_config(cfg)
        L = _lib.lib()
        h = ctypes.c_void_p()
        _lib.check(L.bsml_decoder_create(ctypes.byref(self._c), int(device), ctypes.byref(h)))
        self._h = h
        self.device = torch.device("cuda", device)
        n, ne, na, apc = ctypes.c_int64(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int64()
        _lib.check(L.bsml_decoder_param_count(h, ctypes.byref(n), ctypes.byref(ne), ctypes.byref(na), ctypes.byref(apc)))
        self.n_params, self.n_affine, self.aff_per_clip = n.value, na.value, apc.value
        arr = (_lib.BsmlParamEntry * ne.value)()
        affc = (ctypes.c_int * na.value)()
        rc = L.bsml_decoder_param_table(h, ctypes.cast(arr, ctypes.c_void_p), ne.value, ctypes.cast(affc, ctypes.c_void_p))
        if rc < 0:
            _lib.check(rc)
        self.table = [dict(name=e.name.decode(), offset=e.offset, numel=e.numel, shape=tuple(e.shape[:e.ndim]),
                           trainable=bool(e.trainable)) for e in arr]
        self.aff_C = list(affc)
        self.set_math(math)
        self._last = None

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and _lib._lib is not None:
            _lib.lib().bsml_decoder_destroy(h)
            self._h = None

    def set_math(self, math: str) -> None:
        _lib.check(_lib.lib().bsml_decoder_set_math(self._h, MATH[math]))
        self.math = math

    def set_phase_mode(self, mode: str) -> None:
        """Harmonic-source phase arithmetic: "fp32" (the reference's running
        accumulator, default) or "exact" (double-precision frame phases)."""
        _lib.check(_lib.lib().bsml_decoder_set_phase_mode(self._h, PHASE[mode]))

    def audio_len(self, T: int, frames: int | None = None) -> int:
        c = self.cfg
        if frames is None:
            frames = (2 * T * c["upsample_scale"]) // c["hop"] + 1
        return c["hop"] * (frames - 1)

    def workspace_bytes(self) -> int:
        return int(_lib.lib().bsml_decoder_workspace_bytes(self._h))

    def set_profiling(self, on: bool) -> None:
        _lib.check(_lib.lib().bsml_decoder_set_profiling(self._h, 1 if on else 0))

    # the BSML_PROF_* classes of bsml_decoder_read_profile, in order
    PROFILE_CLASSES = ("conv_tc", "conv_simt", "wgrad_tc", "wgrad_simt", "norm_fwd", "norm_bwd")

    def read_profile(self) -> dict:
        """{class: (ms, algorithmic FLOPs or bytes, launches)} since the last read."""
        buf = (ctypes.c_double * (3 * len(self.PROFILE_CLASSES)))()
        _lib.check(_lib.lib().bsml_decoder_read_profile(self._h, ctypes.cast(buf, ctypes.c_void_p)))
        return {k: (buf[3 * i], buf[3 * i + 1], int(buf[3 * i + 2])) for i, k in enumerate(self.PROFILE_CLASSES)}

    def read_profile_records(self, max_records: int = 4096) -> list:
        """[(class, algorithmic FLOPs or bytes, ms)] per profiled launch, in issue order."""
        buf = (ctypes.c_double * (3 * max_records))()
        n = ctypes.c_int(0)
        _lib.check(_lib.lib().bsml_decoder_read_profile_records(self._h, ctypes.cast(buf, ctypes.c_void_p),
                                                                 max_records, ctypes.byref(n)))
        return [(self.PROFILE_CLASSES[int(buf[3 * i])], buf[3 * i + 1], buf[3 * i + 2]) for i in range(n.value)]

    def forward(self, params, asr, F0, N, style, har=None, aff_in=None, audio=None, aff_out=None):
        params, asr, F0, N, style, har, aff_in = map(_f32, (params, asr, F0, N, style, har, aff_in))
        B, _, T = asr.shape
        frames = 0 if har is None else har.shape[2]
        S = self.audio_len(T, frames if har is not None else None)
        if audio is None:
            audio = torch.empty((B, S), device=self.device, dtype=torch.float32)
        self._last = (B, T)
        # the engine borrows params until the matching backward (like the
        # reference's borrowed weights): keep it alive here
        self._borrowed = params
        _lib.check(_lib.lib().bsml_decoder_forward(
            self._h, B, T, _ptr(params), _ptr(asr), _ptr(F0), _ptr(N), _ptr(style), _ptr(har), frames,
            _ptr(aff_in), _ptr(audio), _ptr(aff_out), _stream()))
        return audio

    def decode(self, params, ref_s, asr, F0, N, audio=None):
        """Kokoro::Impl::decode_back_half (src/kokoro.cpp:352-407), batched: the
        backbone, the harmonic source from F0, the generator and the iSTFT. ref_s
        (B, 2*style_dim): the decoder reads the first style_dim of each row."""
        params, ref_s, asr, F0, N = map(_f32, (params, ref_s, asr, F0, N))
        B, _, T = asr.shape
        if audio is None:
            audio = torch.empty((B, self.audio_len(T)), device=self.device, dtype=torch.float32)
        self._last = (B, T)
        self._borrowed = params
        _lib.check(_lib.lib().bsml_decoder_decode(self._h, B, T, _ptr(params), _ptr(ref_s), ref_s.shape[-1],
                                                  _ptr(asr), _ptr(F0), _ptr(N), _ptr(audio), _stream()))
        return audio

    def backward(self, daudio, grads=None, want_grads=True, want_inputs=True, want_aff=False, d_asr=None,
                 d_style=None):
        """Gradients of the last forward; grads / d_asr / d_style may be given as
        preallocated outputs (nothing is allocated then, e.g. under graph capture)."""
        B, T = self._last
        daudio = _f32(daudio)
        dev = self.device
        if grads is None and want_grads:
            grads = torch.empty(self.n_params, device=dev, dtype=torch.float32)
        if d_asr is None and want_inputs:
            d_asr = torch.empty((B, self.cfg["asr_dim"], T), device=dev)
        if d_style is None and want_inputs:
            d_style = torch.empty((B, self.cfg["style_dim"]), device=dev)
        d_aff = torch.empty(B * self.aff_per_clip, device=dev) if want_aff else None
        _lib.check(_lib.lib().bsml_decoder_backward(self._h, _ptr(daudio), _ptr(grads), _ptr(d_asr),
                                                   _ptr(d_style), _ptr(d_aff), _stream()))
        return dict(grads=grads, d_asr=d_asr, d_style=d_style, d_aff=d_aff)


    # ── the two assemblies on their own (detail::decoder_backbone_* / generator_*)
    def backbone_out_len(self, T: int) -> int:
        n = ctypes.c_int(0)
        _lib.check(_lib.lib().bsml_backbone_out_len(self._h, T, ctypes.byref(n)))
        return n.value

    def forward_backbone(self, params, asr, F0, N, style=None, aff_in=None, gen_in=None, aff_out=None):
        """asr (B, asr_dim, T), F0 / N (B, 2T) -> gen_in (B, init_ch, L_gen)."""
        params, asr, F0, N, style, aff_in = map(_f32, (params, asr, F0, N, style, aff_in))
        B, _, T = asr.shape
        if gen_in is None:
            gen_in = torch.empty((B, self.cfg["init_ch"], self.backbone_out_len(T)), device=self.device)
        self._borrowed = params
        self._last = (B, T)
        st = 0 if style is None else style.shape[-1]
        _lib.check(_lib.lib().bsml_backbone_forward(self._h, B, T, _ptr(params), _ptr(asr), _ptr(F0), _ptr(N),
                                                    _ptr(style), st, _ptr(aff_in), _ptr(gen_in), _ptr(aff_out),
                                                    _stream()))
        return gen_in

    def backward_backbone(self, dgen_in, want_aff=False):
        B, T = self._last
        dev = self.device
        grads = torch.empty(self.n_params, device=dev)
        d_asr = torch.empty((B, self.cfg["asr_dim"], T), device=dev)
        d_style = torch.empty((B, self.cfg["style_dim"]), device=dev)
        d_aff = torch.empty(B * self.aff_per_clip, device=dev) if want_aff else None
        _lib.check(_lib.lib().bsml_backbone_backward(self._h, _ptr(_f32(dgen_in)), _ptr(grads), _ptr(d_asr),
                                                     _ptr(d_style), _ptr(d_aff), _stream()))
        return dict(grads=grads, d_asr=d_asr, d_style=d_style, d_aff=d_aff)

    def forward_generator(self, params, gen_in, har, style=None, aff_in=None, audio=None, aff_out=None):
        """gen_in (B, init_ch, L_in), har (B, har_ch, frames) -> audio (B, hop*(frames-1))."""
        params, gen_in, har, style, aff_in = map(_f32, (params, gen_in, har, style, aff_in))
        B, _, L_in = gen_in.shape
        frames = har.shape[2]
        if audio is None:
            audio = torch.empty((B, self.cfg["hop"] * (frames - 1)), device=self.device)
        self._borrowed = params
        self._last_gen = (B, L_in)
        st = 0 if style is None else style.shape[-1]
        _lib.check(_lib.lib().bsml_generator_forward(self._h, B, L_in, _ptr(params), _ptr(gen_in), _ptr(har),
                                                     frames, _ptr(style), st, _ptr(aff_in), _ptr(audio),
                                                     _ptr(aff_out), _stream()))
        return audio

    def backward_generator(self, daudio, want_aff=False):
        B, L_in = self._last_gen
        dev = self.device
        grads = torch.empty(self.n_params, device=dev)
        dgen = torch.empty((B, self.cfg["init_ch"], L_in), device=dev)
        d_style = torch.empty((B, self.cfg["style_dim"]), device=dev)
        d_aff = torch.empty(B * self.aff_per_clip, device=dev) if want_aff else None
        _lib.check(_lib.lib().bsml_generator_backward(self._h, _ptr(_f32(daudio)), _ptr(grads), _ptr(dgen),
                                                      _ptr(d_style), _ptr(d_aff), _stream()))
        return dict(grads=grads, dgen_in=dgen, d_style=d_style, d_aff=d_aff)


class Block(Decoder):
    """One decoder block on its own over the same engine: ``spec`` =
    dict(kind=1, style_dim, cin, cout, upsample) for an AdainResBlk1d
    (``detail::adain_resblk_1d_forward_train`` / ``_backward``,
    src/kokoro_decoder_backward.h:82-111) or dict(kind=2, style_dim, cin=C, cout=C,
    kernel, dil) for an AdaINResBlock1 (``detail::adain_resblock1_forward_train`` /
    ``_backward``, :125-144). Parameter keys are block-relative."""

    RESBLK1D, RESBLOCK1 = 1, 2

    def __init__(self, spec: dict, device: int = 0, math: str = "fp32"):
        self.spec = dict(spec)
        self.cfg = {"style_dim": spec["style_dim"]}
        self._c = _lib.make_block_spec(spec)
        L = _lib.lib()
        h = ctypes.c_void_p()
        _lib.check(L.bsml_block_create(ctypes.byref(self._c), int(device), ctypes.byref(h)))
        self._h = h
        self.device = torch.device("cuda", device)
        self.n_params, self.table, self.aff_C, self.aff_per_clip = _lib.block_layout(spec)
        self.n_affine = len(self.aff_C)
        self.set_math(math)
        self._last = None

    def out_len(self, L: int) -> int:
        return 2 * L if self.spec["kind"] == self.RESBLK1D and self.spec.get("upsample") else L

    def forward(self, params, x, style=None, aff_in=None, y=None, aff_out=None):
        """x (B, cin, L) -> y (B, cout, out_len(L))."""
        params, x, style, aff_in = map(_f32, (params, x, style, aff_in))
        B, _, L = x.shape
        if y is None:
            y = torch.empty((B, self.spec["cout"], self.out_len(L)), device=self.device, dtype=torch.float32)
        self._last = (B, L)
        self._borrowed = params
        _lib.check(_lib.lib().bsml_block_forward(self._h, B, L, _ptr(params), _ptr(x), _ptr(style), _ptr(aff_in),
                                                 _ptr(y), _ptr(aff_out), _stream()))
        return y

    def backward(self, dy, grads=None, want_grads=True, want_inputs=True, want_aff=False):
        B, L = self._last
        dy = _f32(dy)
        dev = self.device
        if grads is None and want_grads:
            grads = torch.empty(self.n_params, device=dev, dtype=torch.float32)
        dx = torch.empty((B, self.spec["cin"], L), device=dev) if want_inputs else None
        d_style = torch.empty((B, self.spec["style_dim"]), device=dev) if want_inputs else None
        d_aff = torch.empty(B * self.aff_per_clip, device=dev) if want_aff else None
        _lib.check(_lib.lib().bsml_block_backward(self._h, _ptr(dy), _ptr(grads), _ptr(dx), _ptr(d_style),
                                                  _ptr(d_aff), _stream()))
        return dict(grads=grads, dx=dx, d_style=d_style, d_aff=d_aff)


class Graph:
    """A CUDA graph of library calls (bsml_graph_*): every call made on the
    capture stream inside ``with Graph(stream) as g:`` is recorded; ``g.replay()``
    reruns them with the same buffers. Run the sequence once eagerly before
    capturing (workspace planning allocates), pre-allocate every output, and keep
    torch operations out of the captured block."""

    def __init__(self, stream=None):
        self.stream = stream if stream is not None else torch.cuda.Stream()
        self._g = None

    def __enter__(self):
        self._ctx = torch.cuda.stream(self.stream)
        self._ctx.__enter__()
        _lib.check(_lib.lib().bsml_graph_begin(ctypes.c_void_p(self.stream.cuda_stream)))
        return self

    def __exit__(self, et, ev, tb):
        g = ctypes.c_void_p()
        rc = _lib.lib().bsml_graph_end(ctypes.c_void_p(self.stream.cuda_stream), ctypes.byref(g))
        self._ctx.__exit__(et, ev, tb)
        if et is None:
            _lib.check(rc)
            self._g = g
        elif rc == 0 and g.value:
            _lib.lib().bsml_graph_destroy(g)   # the block raised: the partial graph is not kept
        return False

    @property
    def kernels(self) -> int:
        n = ctypes.c_int64()
        _lib.check(_lib.lib().bsml_graph_kernel_count(self._g, ctypes.byref(n)))
        return n.value

    def replay(self, stream=None) -> None:
        s = stream if stream is not None else torch.cuda.current_stream()
        _lib.check(_lib.lib().bsml_graph_launch(self._g, ctypes.c_void_p(s.cuda_stream)))

    def __del__(self):
        if getattr(self, "_g", None) is not None and _lib._lib is not None:
            _lib.lib().bsml_graph_destroy(self._g)
            self._g = None


def l1_loss(audio, target, loss=None, daudio=None):
    audio, target = _f32(audio), _f32(target)
    if loss is None:
        loss = torch.empty(1, device=audio.device)
    if daudio is None:
        daudio = torch.empty_like(audio)
    _lib.check(_lib.lib().bsml_loss_l1(_ptr(audio), _ptr(target), audio.numel(), _ptr(loss), _ptr(daudio), _stream()))
    return loss, daudio


def adam_step(param, grad, m, v, lr, step, beta1=0.9, beta2=0.999, eps=1e-8):
    _lib.check(_lib.lib().bsml_adam_step(_ptr(param), _ptr(grad), _ptr(m), _ptr(v), param.numel(), lr, beta1, beta2,
                                          eps, int(step), _stream()))
