"""Weights and decode inputs on disk, in the safetensors format the reference
loads its converted Kokoro checkpoint from (src/kokoro_modules.cpp:99-125).

* :func:`load_params` fills the flat parameter vector of a :class:`Decoder` (or
  :class:`Block`) from a checkpoint: key = prefix + parameter name, with
  PyTorch weight-norm pairs (``weight_g`` / ``weight_v``) fused on the way as
  the reference's converter does (scripts/convert-kokoro.py:71-110). The reading
  and the fusion run in libbsml_b200.so (``bsml_params_from_safetensors``).
* :func:`save_decode_prep` / :func:`load_decode_prep` / :func:`stack_decode_preps`
  keep the pre-decoder intermediates one clip's training runs over — the fields
  of the reference's ``KokoroDecodePrep`` (include/brosoundml/kokoro.h:132-147):
  ref_s (1, 2*style_dim), asr (hidden, T), F0_pred (2T), N_pred (2T), har
  ((n_fft+2), frames) — as a safetensors file, and stack clips of one length
  into a batch.
* :func:`save_safetensors` writes the format (plain file IO).
"""

from __future__ import annotations

import ctypes
import json
import struct

import numpy as np

from . import _lib

_DT_CODE = {1: "F32", 2: "F16", 3: "BF16", 4: "F64"}
_NP_DT = {np.dtype("float32"): "F32", np.dtype("float16"): "F16", np.dtype("float64"): "F64"}


class SafeTensorsFile:
    """Read access to one safetensors file through the library's reader."""

    def __init__(self, path: str):
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().bsml_st_open(str(path).encode(), ctypes.byref(h)))
        self._h = h
        self.path = str(path)

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and _lib._lib is not None:
            _lib.lib().bsml_st_close(self._h)
            self._h = None

    __del__ = close

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False

    def tensors(self) -> dict:
        """name -> (dtype, shape) in header order."""
        L = _lib.lib()
        n = ctypes.c_int()
        _lib.check(L.bsml_st_count(self._h, ctypes.byref(n)))
        out = {}
        name = ctypes.create_string_buffer(512)
        dt, nd = ctypes.c_int(), ctypes.c_int()
        shape = (ctypes.c_int64 * 8)()
        for i in range(n.value):
            _lib.check(L.bsml_st_info(self._h, i, name, 512, ctypes.byref(dt), ctypes.byref(nd),
                                      ctypes.cast(shape, ctypes.c_void_p)))
            out[name.value.decode()] = (_DT_CODE.get(dt.value, "OTHER"), tuple(shape[:nd.value]))
        return out

    def read(self, name: str) -> np.ndarray:
        """Tensor ``name`` as float32 (from F32, F16, BF16 or F64 data)."""
        shape = self.tensors()[name][1]
        out = np.empty(shape, np.float32)
        _lib.check(_lib.lib().bsml_st_read_f32(self._h, name.encode(), out.ctypes.data_as(ctypes.c_void_p),
                                              out.size))
        return out

    def metadata(self, key: str) -> str:
        buf = ctypes.create_string_buffer(4096)
        _lib.check(_lib.lib().bsml_st_metadata(self._h, key.encode(), buf, 4096))
        return buf.value.decode()


def load_params(model, path: str, prefix: str = "decoder.module.") -> np.ndarray:
    """Flat float32 parameter vector of ``model`` (a Decoder or Block: anything with
    ``table`` and ``n_params``) from the checkpoint at ``path``."""
    n = len(model.table)
    arr = (_lib.BsmlParamEntry * n)()
    for i, e in enumerate(model.table):
        arr[i].name = e["name"].encode()
        arr[i].offset = e["offset"]
        arr[i].numel = e["numel"]
        arr[i].ndim = len(e["shape"])
        for k, d in enumerate(e["shape"]):
            arr[i].shape[k] = d
        arr[i].trainable = 1 if e["trainable"] else 0
    params = np.zeros(model.n_params, np.float32)
    with SafeTensorsFile(path) as f:
        _lib.check(_lib.lib().bsml_params_from_safetensors(f._h, ctypes.cast(arr, ctypes.c_void_p), n,
                                                           prefix.encode(),
                                                           params.ctypes.data_as(ctypes.c_void_p), params.size))
    return params


def save_safetensors(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """Writes name -> numpy array (float32 / float16 / float64) as a safetensors file."""
    header, blobs, off = {}, [], 0
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        if a.dtype not in _NP_DT:
            a = a.astype(np.float32)
        b = a.astype(a.dtype.newbyteorder("<"), copy=False).tobytes()
        header[name] = {"dtype": _NP_DT[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(h)))
        fh.write(h)
        for b in blobs:
            fh.write(b)


# ── KokoroDecodePrep files ────────────────────────────────────────────────────
_PREP_KEYS = ("ref_s", "asr", "F0_pred", "N_pred")


def save_decode_prep(path: str, ref_s, asr, F0_pred, N_pred, har=None) -> None:
    """One clip's decode inputs (KokoroDecodePrep fields) as a safetensors file."""
    asr = np.asarray(asr, np.float32)
    T = asr.shape[-1]
    t = {"ref_s": np.asarray(ref_s, np.float32).reshape(1, -1), "asr": asr.reshape(asr.shape[-2], T),
         "F0_pred": np.asarray(F0_pred, np.float32).reshape(-1), "N_pred": np.asarray(N_pred, np.float32).reshape(-1)}
    if t["F0_pred"].size != 2 * T or t["N_pred"].size != 2 * T:
        raise ValueError("brosoundml: save_decode_prep: F0_pred and N_pred must hold 2*T frames")
    meta = {"format": "KokoroDecodePrep", "total": T, "frames": 0}
    if har is not None:
        har = np.asarray(har, np.float32)
        t["har"] = har.reshape(har.shape[-2], har.shape[-1])
        meta["frames"] = har.shape[-1]
    save_safetensors(path, t, meta)


def load_decode_prep(path: str) -> dict:
    """{ref_s (2S,), asr (hidden, T), F0_pred (2T,), N_pred (2T,), har or None,
    total, frames} from a file written by :func:`save_decode_prep`."""
    with SafeTensorsFile(path) as f:
        names = f.tensors()
        if f.metadata("format") != "KokoroDecodePrep":
            raise ValueError(f"brosoundml: load_decode_prep: {path} is not a KokoroDecodePrep file")
        for k in _PREP_KEYS:
            if k not in names:
                raise ValueError(f"brosoundml: load_decode_prep: missing tensor '{k}' in {path}")
        out = {k: f.read(k) for k in _PREP_KEYS}
        out["ref_s"] = out["ref_s"].reshape(-1)
        out["har"] = f.read("har") if "har" in names else None
        out["total"] = int(f.metadata("total"))
        out["frames"] = int(f.metadata("frames"))
    if out["asr"].shape[1] != out["total"] or out["F0_pred"].size != 2 * out["total"]:
        raise ValueError(f"brosoundml: load_decode_prep: inconsistent shapes in {path}")
    return out


def stack_decode_preps(preps: list) -> dict:
    """Batch of clips of one length: ref_s (B, 2S), asr (B, hidden, T), F0 / N
    (B, 2T), har (B, har_ch, frames) or None (then every clip must lack it)."""
    if not preps:
        raise ValueError("brosoundml: stack_decode_preps: no clips")
    T = preps[0]["total"]
    if any(p["total"] != T for p in preps):
        raise ValueError("brosoundml: stack_decode_preps: clips differ in length (T)")
    has_har = [p["har"] is not None for p in preps]
    if any(has_har) and not all(has_har):
        raise ValueError("brosoundml: stack_decode_preps: har given for some clips only")
    out = {"ref_s": np.stack([p["ref_s"] for p in preps]), "asr": np.stack([p["asr"] for p in preps]),
           "F0": np.stack([p["F0_pred"] for p in preps]), "N": np.stack([p["N_pred"] for p in preps]),
           "har": np.stack([p["har"] for p in preps]) if all(has_har) else None, "total": T}
    return out
