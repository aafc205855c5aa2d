"""CPU restatement of the DecoderLora adapter and gate math, float64 numpy.

TEST INFRASTRUCTURE ONLY: the checker for brosoundml_b200's DecoderLora
(bsml_lora_*); the product never imports this module.

Follows the reference's src/decoder_lora.cpp:
  gate (:30-78):      g = W2 tanh(W1 v), no biases; dW2 += dG act^T, dW1 += ((W2^T dG)(1-act^2)) v^T
  adapters (:184-207) through brotensor lora_forward / lora_backward (brotensor is
  not vendored; its contract as the reference uses it):
      h = A s,  hg = g * h,  (gamma ; beta) = W s + b + scale * B hg
      dB += scale * dY hg^T,  dhg = scale * B^T dY,  dA += (dhg * g) s^T,  dG += dhg * h
  composition (:211-296): every AdaIN's (gamma, beta) from its adapter, the decoder in
  reference mode, the affine gradients back through the adapters into one shared dG.
Batched here: clip b has its own style s_b and condition v_b (the reference has one clip).

Parity status: unpinned by reference artefacts (no golden LoRA vectors exist); pinned by
finite differences (tests/test_lora_cpu.py).
"""

from __future__ import annotations

import numpy as np

IN_DIM, HIDDEN = 3, 16


class LoraLayout:
    """Offsets of the flat LoRA parameter vector: gate W1 [16][3], gate W2 [rank][16],
    then per adapter (DecoderLora::adapters() order) A [rank][S], B [2C][rank]."""

    def __init__(self, aff_C, rank: int, style_dim: int):
        self.aff_C, self.rank, self.S = list(aff_C), rank, style_dim
        self.off_W1 = 0
        self.off_W2 = HIDDEN * IN_DIM
        off = self.off_W2 + rank * HIDDEN
        self.off_A, self.off_B = [], []
        for C in self.aff_C:
            self.off_A.append(off)
            off += rank * style_dim
            self.off_B.append(off)
            off += 2 * C * rank
        self.n_params = off
        self.aff_base = np.concatenate([[0], np.cumsum([2 * c for c in self.aff_C])[:-1]]).astype(int)
        self.aff_per_clip = int(sum(2 * c for c in self.aff_C))

    def W1(self, p):
        return p[self.off_W1:self.off_W1 + HIDDEN * IN_DIM].reshape(HIDDEN, IN_DIM)

    def W2(self, p):
        return p[self.off_W2:self.off_W2 + self.rank * HIDDEN].reshape(self.rank, HIDDEN)

    def A(self, p, a):
        return p[self.off_A[a]:self.off_A[a] + self.rank * self.S].reshape(self.rank, self.S)

    def B(self, p, a):
        return p[self.off_B[a]:self.off_B[a] + 2 * self.aff_C[a] * self.rank].reshape(2 * self.aff_C[a], self.rank)


def fc_offsets(table):
    """(weight, bias) offsets of every AdaIN fc, in adapters() order (= table order)."""
    w = [e for e in table if e["name"].endswith(".fc.weight")]
    b = [e for e in table if e["name"].endswith(".fc.bias")]
    return [(x["offset"], y["offset"]) for x, y in zip(w, b)]


def gate_forward(lay: LoraLayout, lp, cond):
    act = np.tanh(cond @ lay.W1(lp).T)            # (B, hidden)
    return act, act @ lay.W2(lp).T                # g: (B, rank)


def affines(lay: LoraLayout, fc, params, lp, style, cond, scale):
    """Packed [a][B][2C] (gamma ; beta) of every AdaIN for every clip, and the caches."""
    B = style.shape[0]
    act, g = gate_forward(lay, lp, cond)
    aff = np.zeros(B * lay.aff_per_clip)
    hs = []
    for a, C in enumerate(lay.aff_C):
        wo, bo = fc[a]
        W = params[wo:wo + 2 * C * lay.S].reshape(2 * C, lay.S)
        b = params[bo:bo + 2 * C]
        h = style @ lay.A(lp, a).T                # (B, rank)
        y = style @ W.T + b + scale * (g * h) @ lay.B(lp, a).T
        aff[B * lay.aff_base[a]:B * lay.aff_base[a] + B * 2 * C] = y.reshape(-1)
        hs.append(h)
    return aff, (act, g, hs)


def backward(lay: LoraLayout, lp, style, cond, scale, d_aff, cache):
    """LoRA + gate gradients (flat, the parameter layout) from the packed affine gradients."""
    act, g, hs = cache
    B = style.shape[0]
    grad = np.zeros(lay.n_params)
    dG = np.zeros_like(g)
    for a, C in enumerate(lay.aff_C):
        dY = d_aff[B * lay.aff_base[a]:B * lay.aff_base[a] + B * 2 * C].reshape(B, 2 * C)
        h = hs[a]
        hg = g * h
        grad[lay.off_B[a]:lay.off_B[a] + 2 * C * lay.rank] += (scale * dY.T @ hg).reshape(-1)
        dhg = scale * dY @ lay.B(lp, a)          # (B, rank)
        grad[lay.off_A[a]:lay.off_A[a] + lay.rank * lay.S] += ((dhg * g).T @ style).reshape(-1)
        dG += dhg * h
    grad[lay.off_W2:lay.off_W2 + lay.rank * HIDDEN] += (dG.T @ act).reshape(-1)
    dpre = (dG @ lay.W2(lp)) * (1.0 - act * act)
    grad[lay.off_W1:lay.off_W1 + HIDDEN * IN_DIM] += (dpre.T @ cond).reshape(-1)
    return grad


def run(oracle, lay: LoraLayout, params, lp, asr, F0, N, style, cond, scale, har=None, daudio=None):
    """Forward (and backward when daudio is given) of the decoder under the adapters, float64."""
    fc = fc_offsets(oracle.table)
    aff, cache = affines(lay, fc, params.astype(np.float64), lp.astype(np.float64), style.astype(np.float64),
                         cond.astype(np.float64), scale)
    out = oracle.run(params, asr, F0, N, style, har=har, aff_in=aff, daudio=daudio, dtype=np.float64)
    res = {"audio": out["audio"], "aff": aff}
    if daudio is not None:
        res["grads"] = backward(lay, lp.astype(np.float64), style.astype(np.float64), cond.astype(np.float64),
                                scale, out["d_aff"], cache)
    return res


def read_elra1(path: str):
    """Independent reader of the ELRA1 checkpoint (src/decoder_lora.cpp:324-396):
    returns (rank, style_dim, scale, hidden, W1, W2, [(C, A, B), ...])."""
    with open(path, "rb") as f:
        data = f.read()
    if data[:8] != b"ELRA1\0\0\0":
        raise ValueError("bad magic")
    pos = 8

    def i32():
        nonlocal pos
        v = int(np.frombuffer(data, "<i4", 1, pos)[0])
        pos += 4
        return v

    def tensor():
        nonlocal pos
        r, c = i32(), i32()
        t = np.frombuffer(data, "<f4", r * c, pos).reshape(r, c).copy()
        pos += 4 * r * c
        return t

    rank, sd = i32(), i32()
    scale = float(np.frombuffer(data, "<f4", 1, pos)[0])
    pos += 4
    hidden = i32()
    W1, W2 = tensor(), tensor()
    ads = []
    while pos < len(data) and data[pos:pos + 8] != b"ELRSTATE":   # optimiser state may follow
        C = i32()
        A, B = tensor(), tensor()
        ads.append((C, A, B))
    return rank, sd, scale, hidden, W1, W2, ads


# ── conv-weight LoRA (no reference counterpart) ───────────────────────────────
class ConvLoraLayout:
    """Every 3-d ``*.weight`` of the decoder (Conv1d / ConvTranspose1d), viewed [d0][d1*k];
    flat LoRA vector: per weight A [rank][d1*k] then B [d0][rank]."""

    def __init__(self, table, rank: int):
        self.rank = rank
        self.ws = []
        off = 0
        for e in table:
            if len(e["shape"]) != 3 or not e["name"].endswith(".weight"):
                continue
            rows, cols = e["shape"][0], e["shape"][1] * e["shape"][2]
            self.ws.append(dict(w=e["offset"], rows=rows, cols=cols, offA=off, offB=off + rank * cols))
            off += rank * cols + rows * rank
        self.n_params = off


def conv_lora_fold(lay: ConvLoraLayout, params, lp, scale):
    eff = params.astype(np.float64).copy()
    for w in lay.ws:
        A = lp[w["offA"]:w["offA"] + lay.rank * w["cols"]].reshape(lay.rank, w["cols"])
        B = lp[w["offB"]:w["offB"] + w["rows"] * lay.rank].reshape(w["rows"], lay.rank)
        eff[w["w"]:w["w"] + w["rows"] * w["cols"]] += scale * (B @ A).reshape(-1)
    return eff


def conv_lora_grads(lay: ConvLoraLayout, lp, dW_full, scale):
    g = np.zeros(lay.n_params)
    for w in lay.ws:
        A = lp[w["offA"]:w["offA"] + lay.rank * w["cols"]].reshape(lay.rank, w["cols"])
        B = lp[w["offB"]:w["offB"] + w["rows"] * lay.rank].reshape(w["rows"], lay.rank)
        dW = dW_full[w["w"]:w["w"] + w["rows"] * w["cols"]].reshape(w["rows"], w["cols"])
        g[w["offA"]:w["offA"] + lay.rank * w["cols"]] = (scale * B.T @ dW).reshape(-1)
        g[w["offB"]:w["offB"] + w["rows"] * lay.rank] = (scale * dW @ A.T).reshape(-1)
    return g


def conv_lora_run(oracle, lay: ConvLoraLayout, params, lp, asr, F0, N, style, scale, har=None, daudio=None):
    eff = conv_lora_fold(lay, params, lp.astype(np.float64), scale)
    out = oracle.run(eff, asr, F0, N, style, har=har, daudio=daudio, dtype=np.float64)
    res = {"audio": out["audio"]}
    if daudio is not None:
        res["grads"] = conv_lora_grads(lay, lp.astype(np.float64), out["grads"], scale)
    return res
