"""Independent PyTorch-autograd restatement of the Kokoro decoder (CPU).

TEST INFRASTRUCTURE ONLY (second oracle). It is written from the PyTorch
definitions the upstream Kokoro model uses — F.conv1d, F.conv_transpose1d,
F.instance_norm (eps 1e-5, biased variance), torch.istft(center=True, periodic
Hann), F.pad(reflect) — following the composition of the reference's
src/kokoro_decoder_backward.cpp (forward_train assemblies) and
src/kokoro_modules.cpp:1087-1141 / 1197-1231 / 1400-1552. Gradients come from
autograd, so agreement with the hand-written C++ oracle pins both.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


def hann(n: int, dtype) -> torch.Tensor:
    # Same float32 arithmetic as kokoro_decoder_backward.cpp:581-588.
    i = torch.arange(n, dtype=torch.float32)
    w = 0.5 - 0.5 * torch.cos(6.28318530717958647692 * i / n)
    return w.to(dtype)


class TorchDecoder:
    def __init__(self, cfg: dict, table, params: np.ndarray, dtype=torch.float64, device=None):
        self.cfg = cfg
        self.dtype = dtype
        self.p = {}
        for e in table:
            t = torch.tensor(params[e["offset"]:e["offset"] + e["numel"]], dtype=dtype,
                             device=device).reshape(e["shape"])
            t.requires_grad_(e["trainable"])
            self.p[e["name"]] = t
        self.table = table

    def grads_flat(self, n_params: int) -> np.ndarray:
        g = np.zeros(n_params, np.float64)
        for e in self.table:
            t = self.p[e["name"]]
            if t.grad is not None:
                g[e["offset"]:e["offset"] + e["numel"]] = t.grad.detach().reshape(-1).cpu().numpy()
        return g

    # ── pieces
    def affine(self, prefix, style, aff_override):
        if aff_override is not None:
            gb = aff_override.pop(0)
        else:
            gb = F.linear(style, self.p[prefix + ".fc.weight"], self.p[prefix + ".fc.bias"])
        self.aff_list.append(gb)
        return gb

    def adain(self, x, prefix, style, aff_override):
        gb = self.affine(prefix, style, aff_override)
        C = x.shape[1]
        g, b = gb[:, :C, None], gb[:, C:, None]
        return (1 + g) * F.instance_norm(x, eps=1e-5) + b

    def blk(self, x, pre, style, cin, cout, up, aff):
        p = self.p
        r = F.leaky_relu(self.adain(x, pre + ".norm1", style, aff), 0.2)
        if up:
            r = F.conv_transpose1d(r, p[pre + ".pool.weight"], p[pre + ".pool.bias"], stride=2, padding=1,
                                   output_padding=1, groups=cin)
        c1 = F.conv1d(r, p[pre + ".conv1.weight"], p[pre + ".conv1.bias"], padding=1)
        n2 = F.leaky_relu(self.adain(c1, pre + ".norm2", style, aff), 0.2)
        c2 = F.conv1d(n2, p[pre + ".conv2.weight"], p[pre + ".conv2.bias"], padding=1)
        sc = x.repeat_interleave(2, dim=2) if up else x
        if cin != cout:
            sc = F.conv1d(sc, p[pre + ".conv1x1.weight"])
        return (c2 + sc) / np.sqrt(2.0)

    def rb1(self, x, pre, style, k, dil, aff):
        p = self.p
        # adapter order: adain1[0..2] then adain2[0..2] (decoder_lora.cpp:128-135)
        gbs1 = [self.affine(f"{pre}.adain1.{i}", style, aff) for i in range(3)]
        gbs2 = [self.affine(f"{pre}.adain2.{i}", style, aff) for i in range(3)]
        C = x.shape[1]
        for i in range(3):
            a = p[f"{pre}.alpha1.{i}"]
            xt = (1 + gbs1[i][:, :C, None]) * F.instance_norm(x, eps=1e-5) + gbs1[i][:, C:, None]
            xt = xt + torch.sin(a * xt) ** 2 / a
            xt = F.conv1d(xt, p[f"{pre}.convs1.{i}.weight"], p[f"{pre}.convs1.{i}.bias"],
                          padding=(k * dil[i] - dil[i]) // 2, dilation=dil[i])
            a = p[f"{pre}.alpha2.{i}"]
            xt = (1 + gbs2[i][:, :C, None]) * F.instance_norm(xt, eps=1e-5) + gbs2[i][:, C:, None]
            xt = xt + torch.sin(a * xt) ** 2 / a
            xt = F.conv1d(xt, p[f"{pre}.convs2.{i}.weight"], p[f"{pre}.convs2.{i}.bias"], padding=(k - 1) // 2)
            x = xt + x
        return x

    def forward(self, asr, F0, N, style, har, aff_override=None):
        """All inputs torch tensors; aff_override: list of per-AdaIN (B, 2C) tensors (reference mode)."""
        c, p = self.cfg, self.p
        aff = list(aff_override) if aff_override is not None else None
        self.aff_list = []
        T = asr.shape[2]
        F0dn = F.conv1d(F0[:, None, :], p["F0_conv.weight"], p["F0_conv.bias"], stride=2, padding=1)
        Ndn = F.conv1d(N[:, None, :], p["N_conv.weight"], p["N_conv.bias"], stride=2, padding=1)
        asr_res = F.conv1d(asr, p["asr_res.0.weight"], p["asr_res.0.bias"])
        x = self.blk(torch.cat([asr, F0dn, Ndn], 1), "encode", style, c["asr_dim"] + 2, c["enc_dim"], False, aff)
        res = True
        for i in range(c["n_decode"]):
            cin = x.shape[1] + (c["asr_res_dim"] + 2 if res else 0)
            if res:
                x = torch.cat([x, asr_res, F0dn, Ndn], 1)
            up = i == c["upsample_block"]
            x = self.blk(x, f"decode.{i}", style, cin, c["dec_out"][i], up, aff)
            if up:
                res = False
        U, K = c["n_ups"], c["n_kernels"]
        # affine order: all noise_res first, then resblocks (DecoderLora::adapters())
        for i in range(U):
            a = F.leaky_relu(x, 0.1)
            xs = F.conv1d(har, p[f"generator.noise_convs.{i}.weight"], p[f"generator.noise_convs.{i}.bias"],
                          stride=c["noise_stride"][i], padding=c["noise_pad"][i])
            src = self.rb1(xs, f"generator.noise_res.{i}", style, c["nr_kernel"][i], c["nr_dil"][i], aff)
            kk, s = c["ups_kernel"][i], c["ups_rate"][i]
            u = F.conv_transpose1d(a, p[f"generator.ups.{i}.weight"], p[f"generator.ups.{i}.bias"], stride=s,
                                   padding=(kk - s) // 2)
            if i == U - 1:
                u = F.pad(u, (1, 0), mode="reflect")
            m = u + src
            xs_sum = 0
            for j in range(K):
                xs_sum = xs_sum + self.rb1(m, f"generator.resblocks.{i * K + j}", style, c["rb_kernel"][j],
                                           c["rb_dil"][j], aff)
            x = xs_sum / K
        x = F.leaky_relu(x, 0.01)
        post = F.conv1d(x, p["generator.conv_post.weight"], p["generator.conv_post.bias"],
                        padding=(c["post_kernel"] - 1) // 2)
        nf = c["n_fft"] // 2 + 1
        mag = torch.exp(post[:, :nf])
        ph = torch.sin(post[:, nf:])
        spec = torch.complex(mag * torch.cos(ph), mag * torch.sin(ph))
        audio = torch.istft(spec, c["n_fft"], c["hop"], win_length=c["n_fft"], window=hann(c["n_fft"], self.dtype),
                            center=True)
        return audio

    def reorder_affines(self):
        """self.aff_list is in forward-call order; the oracle's packing order is
        encode, decode..., noise_res..., resblocks... — the forward visits the
        generator stage by stage (noise_res[i] then resblocks of stage i), so
        regroup into the adapter order."""
        c = self.cfg
        nb = 2 * (1 + c["n_decode"])
        bb = self.aff_list[:nb]
        gen = self.aff_list[nb:]
        U, K = c["n_ups"], c["n_kernels"]
        noise, res = [], []
        q = 0
        for i in range(U):
            noise += gen[q:q + 6]
            q += 6
            for j in range(K):
                res += gen[q:q + 6]
                q += 6
        return bb + noise + res


def harmonic_source_torch(F0: np.ndarray, lw: np.ndarray, lb: np.ndarray, cfg: dict) -> np.ndarray:
    """Harmonic source restated in float64 (closed-form phase, torch.stft).
    Phases agree with the reference's fp32 running sum only to rounding."""
    B, Fr = F0.shape
    ups = cfg["upsample_scale"]
    S = Fr * ups
    f0 = np.repeat(F0.astype(np.float64), ups, axis=1)  # (B, S)
    h = np.arange(1, cfg["harmonic_num"] + 2, dtype=np.float64)
    omega = 2 * np.pi * f0[:, :, None] * h[None, None, :] / cfg["sample_rate"]
    phase = np.mod(np.cumsum(omega, axis=1), 2 * np.pi)
    uv = (f0 > 0).astype(np.float64)[:, :, None]
    sines = np.sin(phase) * 0.1 * uv
    merged = np.tanh(sines @ lw.reshape(-1).astype(np.float64) + float(lb.reshape(-1)[0]))
    x = torch.tensor(merged)
    spec = torch.stft(x, cfg["n_fft"], cfg["hop"], win_length=cfg["n_fft"], window=hann(cfg["n_fft"], torch.float64),
                      center=True, pad_mode="reflect", return_complex=True)
    return torch.cat([spec.abs(), spec.angle()], 1).numpy()
