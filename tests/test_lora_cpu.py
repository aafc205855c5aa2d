"""DecoderLora maths on the CPU (float64 oracle, no GPU): finite-difference checks
of the adapter and gate gradients through the whole miniature decoder (the
reference's LoRA / gate FD checks, tests/test_kokoro_decoder_backward.cpp:553-560,
tests/test_decoder_lora.cpp:52-102) and the gate's zero-init property."""

import numpy as np

from brosoundml_b200 import config, synth
from oracle import lora_oracle as lo
from oracle.oracle import Oracle
from tests.helpers import random_params

B, T, FRAMES, RANK, SCALE = 2, 4, 33, 4, 2.0


def _setup(seed=0):
    cfg = config.miniature()
    o = Oracle(cfg)
    lay = lo.LoraLayout(o.aff_C, RANK, cfg["style_dim"])
    rng = np.random.default_rng(seed)
    p = random_params(o.table, o.n_params, 11)
    lp = rng.uniform(-0.5, 0.5, lay.n_params)
    x = {k: v.astype(np.float64) for k, v in synth.make_inputs(cfg, B, T, 1).items()}
    har = rng.uniform(-0.4, 0.4, (B, cfg["har_ch"], FRAMES))
    cond = rng.normal(0, 1, (B, lo.IN_DIM))
    tgt = rng.uniform(-0.3, 0.3, (B, cfg["hop"] * (FRAMES - 1)))
    return o, lay, p, lp, x, har, cond, tgt


def test_lora_grads_directional_fd():
    o, lay, p, lp, x, har, cond, tgt = _setup()

    def loss(q):
        a = lo.run(o, lay, p, q, x["asr"], x["F0"], x["N"], x["style"], cond, SCALE, har=har)["audio"]
        return 0.5 * float(((a - tgt) ** 2).sum())

    a = lo.run(o, lay, p, lp, x["asr"], x["F0"], x["N"], x["style"], cond, SCALE, har=har)["audio"]
    g = lo.run(o, lay, p, lp, x["asr"], x["F0"], x["N"], x["style"], cond, SCALE, har=har, daudio=a - tgt)["grads"]
    rng = np.random.default_rng(7)
    groups = {"W1": [slice(lay.off_W1, lay.off_W1 + lo.HIDDEN * lo.IN_DIM)],
              "W2": [slice(lay.off_W2, lay.off_W2 + RANK * lo.HIDDEN)],
              "A": [slice(lay.off_A[i], lay.off_A[i] + RANK * lay.S) for i in range(len(lay.aff_C))],
              "B": [slice(lay.off_B[i], lay.off_B[i] + 2 * c * RANK) for i, c in enumerate(lay.aff_C)]}
    for key, sls in groups.items():
        v = np.zeros_like(lp)
        for s in sls:
            v[s] = rng.uniform(-1, 1, s.stop - s.start)
        h = 1e-6
        fd = (loss(lp + h * v) - loss(lp - h * v)) / (2 * h)
        an = float((g * v).sum())
        assert abs(an - fd) <= 1e-7 + 1e-5 * abs(fd), (key, an, fd)


def test_gate_zero_w2_is_the_base_decoder():
    """W2 = 0 (the state DecoderLora::make leaves the gate in) makes g(v) = 0 for any v:
    the adapters add nothing and every AdaIN gets fc(style)."""
    o, lay, p, lp, x, har, cond, tgt = _setup(1)
    lp[lay.off_W2:lay.off_W2 + RANK * lo.HIDDEN] = 0.0
    r = lo.run(o, lay, p, lp, x["asr"], x["F0"], x["N"], x["style"], cond, SCALE, har=har)
    base = o.run(p, x["asr"], x["F0"], x["N"], x["style"], har=har, dtype=np.float64)
    assert np.abs(r["audio"] - base["audio"]).max() <= 1e-12 * max(1.0, np.abs(base["audio"]).max())
    _, gv = lo.gate_forward(lay, lp, cond)
    assert np.all(gv == 0.0)


def test_elra1_reader_roundtrip(tmp_path):
    """The test-side ELRA1 reader against a file written by the format's rules."""
    lay = lo.LoraLayout([3, 5], 2, 4)
    lp = np.arange(lay.n_params, dtype=np.float32)
    path = tmp_path / "x.elra"
    with open(path, "wb") as f:
        f.write(b"ELRA1\0\0\0")
        f.write(np.array([2, 4], "<i4").tobytes())
        f.write(np.array([1.5], "<f4").tobytes())
        f.write(np.array([lo.HIDDEN], "<i4").tobytes())
        for t in (lay.W1(lp), lay.W2(lp)):
            f.write(np.array(t.shape, "<i4").tobytes() + t.astype("<f4").tobytes())
        for a, C in enumerate(lay.aff_C):
            f.write(np.array([C], "<i4").tobytes())
            for t in (lay.A(lp, a), lay.B(lp, a)):
                f.write(np.array(t.shape, "<i4").tobytes() + t.astype("<f4").tobytes())
    rank, sd, scale, hidden, W1, W2, ads = lo.read_elra1(str(path))
    assert (rank, sd, scale, hidden) == (2, 4, 1.5, lo.HIDDEN)
    assert np.array_equal(W1, lay.W1(lp)) and np.array_equal(W2, lay.W2(lp))
    assert [c for c, _, _ in ads] == [3, 5]
    assert np.array_equal(ads[1][2], lay.B(lp, 1))


def test_conv_lora_grads_directional_fd():
    """Conv-weight LoRA (config 3): dA, dB from the decoder's weight gradients against
    finite differences of the adapted miniature decoder."""
    o, lay_, p, lp_, x, har, cond, tgt = _setup(3)
    lay = lo.ConvLoraLayout(o.table, RANK)
    assert len(lay.ws) > 0
    lp = np.random.default_rng(8).normal(0, 0.05, lay.n_params)

    def loss(q):
        a = lo.conv_lora_run(o, lay, p, q, x["asr"], x["F0"], x["N"], x["style"], SCALE, har=har)["audio"]
        return 0.5 * float(((a - tgt) ** 2).sum())

    a = lo.conv_lora_run(o, lay, p, lp, x["asr"], x["F0"], x["N"], x["style"], SCALE, har=har)["audio"]
    g = lo.conv_lora_run(o, lay, p, lp, x["asr"], x["F0"], x["N"], x["style"], SCALE, har=har, daudio=a - tgt)["grads"]
    rng = np.random.default_rng(9)
    for part in ("A", "B"):
        v = np.zeros_like(lp)
        for w in lay.ws:
            s = slice(w["offA"], w["offB"]) if part == "A" else slice(w["offB"], w["offB"] + w["rows"] * RANK)
            v[s] = rng.uniform(-1, 1, s.stop - s.start)
        h = 1e-6
        fd = (loss(lp + h * v) - loss(lp - h * v)) / (2 * h)
        an = float((g * v).sum())
        assert abs(an - fd) <= 1e-7 + 1e-5 * abs(fd), (part, an, fd)
