"""Seeded synthetic inputs with the shapes and value distributions BASELINE.json
names for the Kokoro decoder configs (no public dataset is involved):

  weights N(0, 0.02) (every conv / convT / fc weight and bias, l_linear), Snake alpha = 1
  asr   (B, 512, T)  N(0, 1)
  F0    (B, 2T)      U(80, 300) Hz with a seeded 70 % voiced mask (0 where unvoiced)
  N     (B, 2T)      N(0, 1)
  style (B, 128)     N(0, 1)
  target (B, S)      U(-0.1, 0.1); loss = mean |audio - target|

Generated with numpy's PCG64 so the CPU oracle, the PyTorch model and the CUDA
path all consume identical bytes.
"""

from __future__ import annotations

import numpy as np

from . import config as _config


def init_params(table, n_params: int, seed: int = 0, std: float = 0.02) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    p = np.zeros(n_params, np.float32)
    for e in table:
        o, n = e["offset"], e["numel"]
        if ".alpha" in e["name"]:
            p[o:o + n] = 1.0
        else:
            p[o:o + n] = rng.normal(0.0, std, n).astype(np.float32)
    return p


def make_inputs(cfg: dict, B: int, T: int, seed: int = 1):
    rng = np.random.Generator(np.random.PCG64(seed))
    asr = rng.normal(0.0, 1.0, (B, cfg["asr_dim"], T)).astype(np.float32)
    f0 = rng.uniform(80.0, 300.0, (B, 2 * T)).astype(np.float32)
    voiced = rng.uniform(0.0, 1.0, (B, 2 * T)) < 0.7
    F0 = np.where(voiced, f0, 0.0).astype(np.float32)
    N = rng.normal(0.0, 1.0, (B, 2 * T)).astype(np.float32)
    style = rng.normal(0.0, 1.0, (B, cfg["style_dim"])).astype(np.float32)
    return dict(asr=asr, F0=F0, N=N, style=style)


def make_target(cfg: dict, B: int, T: int, seed: int = 2) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    S = _config.audio_len(cfg, T)
    return rng.uniform(-0.1, 0.1, (B, S)).astype(np.float32)


def l1_grad(audio: np.ndarray, target: np.ndarray):
    """loss = mean |a - t|; d loss / d a = sign(a - t) / numel."""
    d = audio - target
    return float(np.abs(d).mean()), (np.sign(d) / d.size).astype(audio.dtype)
