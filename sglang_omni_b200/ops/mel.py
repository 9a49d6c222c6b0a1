"""Whisper-style log-mel front-end (n_fft 400, hop 160, 128 Slaney mel bins,
log10, clamp to max-8, (x+4)/4) for 16 kHz audio.

GPU path: framing (reflect-padded, Hann window) then the DFT as a GEMM against
a precomputed [cos; sin] basis and the mel projection as a second GEMM, both
on the tcgen05 kernel (fp32 accumulation).  CPU path: torch.stft, the oracle.
Reference counterpart: the HF WhisperFeatureExtractor inside the Qwen3-Omni
processor (sglang_omni/models/qwen3_omni/components/preprocessor.py:249-257)
and ming's whisper.log_mel_spectrogram
(sglang_omni/models/ming_omni/components/preprocessor.py:43-72).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from .gemm import linear

N_FFT, HOP, SR = 400, 160, 16000


def _hz_to_mel(f):
    f = np.asarray(f, dtype=np.float64)
    f_sp = 200.0 / 3
    mels = f / f_sp
    min_log_hz = 1000.0
    min_log_mel = min_log_hz / f_sp
    logstep = math.log(6.4) / 27.0
    return np.where(f >= min_log_hz, min_log_mel + np.log(np.maximum(f, 1e-10) / min_log_hz) / logstep, mels)


def _mel_to_hz(m):
    m = np.asarray(m, dtype=np.float64)
    f_sp = 200.0 / 3
    freqs = f_sp * m
    min_log_hz = 1000.0
    min_log_mel = min_log_hz / f_sp
    logstep = math.log(6.4) / 27.0
    return np.where(m >= min_log_mel, min_log_hz * np.exp(logstep * (m - min_log_mel)), freqs)


def mel_filters(n_mels: int = 128, n_fft: int = N_FFT, sr: int = SR) -> np.ndarray:
    """Slaney-scale, Slaney-normalised triangular filters [n_mels, n_fft//2 + 1]."""
    fft_freqs = np.linspace(0, sr / 2, n_fft // 2 + 1)
    mel_pts = _mel_to_hz(np.linspace(_hz_to_mel(0.0), _hz_to_mel(sr / 2), n_mels + 2))
    fdiff = np.diff(mel_pts)
    ramps = mel_pts[:, None] - fft_freqs[None, :]
    lower = -ramps[:-2] / fdiff[:-1, None]
    upper = ramps[2:] / fdiff[1:, None]
    w = np.maximum(0, np.minimum(lower, upper))
    enorm = 2.0 / (mel_pts[2:n_mels + 2] - mel_pts[:n_mels])
    return (w * enorm[:, None]).astype(np.float32)


class LogMel:
    def __init__(self, n_mels: int = 128, device="cpu"):
        self.n_mels = n_mels
        self.device = torch.device(device)
        self.filters = torch.from_numpy(mel_filters(n_mels)).to(self.device)
        self.window = torch.hann_window(N_FFT, periodic=True).to(self.device)
        if self.device.type == "cuda":
            n = torch.arange(N_FFT, dtype=torch.float64)
            k = torch.arange(N_FFT // 2 + 1, dtype=torch.float64)
            ang = 2 * math.pi * k[:, None] * n[None, :] / N_FFT
            win = torch.hann_window(N_FFT, periodic=True, dtype=torch.float64)
            basis = torch.zeros(512, 400, dtype=torch.float64)
            basis[:402] = torch.cat([torch.cos(ang) * win, -torch.sin(ang) * win], 0)  # [402, 400]
            # bf16 hi/lo split of the basis: with the input split the same way one
            # GEMM over K = [x_hi | x_hi | x_lo] . [b_hi | b_lo | b_hi] keeps ~16-bit accuracy
            b_hi = basis.to(torch.bfloat16)
            b_lo = (basis - b_hi.double()).to(torch.bfloat16)
            self.basis = torch.cat([b_hi, b_lo, b_hi], 1).to(self.device)  # [512, 1200]
            fb = torch.zeros(n_mels, 208, dtype=torch.float32)
            fb[:, :201] = self.filters.cpu()
            self.fb = fb.to(self.device, torch.bfloat16)

    def __call__(self, audio: torch.Tensor) -> torch.Tensor:
        """audio: float [N] at 16 kHz -> log-mel [n_mels, N // 160]."""
        if self.device.type != "cuda":
            audio = audio.to(self.device, torch.float32)
            st = torch.stft(audio, N_FFT, HOP, window=self.window, return_complex=True)
            mag = st[..., :-1].abs() ** 2
            mel = self.filters @ mag
            log_spec = torch.clamp(mel, min=1e-10).log10()
            log_spec = torch.maximum(log_spec, log_spec.max() - 8.0)
            return (log_spec + 4.0) / 4.0
        return self.batch([audio])[0]

    def batch(self, audios: list[torch.Tensor]) -> list[torch.Tensor]:
        """Log-mel of several waveforms: waveforms of equal length are framed, scaled and
        projected together (one DFT GEMM and one mel GEMM per length), with per-waveform bf16
        range scales (frame peak before the DFT, power peak before the mel projection) kept
        on the device: no host round trip and no per-waveform kernels."""
        if self.device.type != "cuda":
            return [self(a) for a in audios]
        # one pinned host buffer and one copy for every waveform of the batch (a pageable copy
        # per waveform blocks the host thread each time)
        host = [a.reshape(-1).to(torch.float32) for a in audios]
        if all(not h.is_cuda for h in host):
            flat = torch.cat(host).pin_memory().to(self.device, non_blocking=True)
            dev_waves = list(torch.split(flat, [h.numel() for h in host]))
        else:
            dev_waves = [h.to(self.device, non_blocking=True) for h in host]
        groups: dict[int, list[int]] = {}
        for i, w in enumerate(dev_waves):
            groups.setdefault(w.numel(), []).append(i)
        out: list = [None] * len(dev_waves)
        for idxs in groups.values():
            for i, m in zip(idxs, self._group(torch.stack([dev_waves[i] for i in idxs]))):
                out[i] = m
        return out

    def _group(self, x: torch.Tensor) -> torch.Tensor:
        """x [b, N] equal-length waveforms -> [b, n_mels, N // 160]."""
        b = x.shape[0]
        xp = torch.nn.functional.pad(x[:, None], (N_FFT // 2, N_FFT // 2), mode="reflect")[:, 0]
        fr = xp.unfold(1, N_FFT, HOP)[:, :-1]                       # [b, T, 400]
        T = fr.shape[1]
        # scale into bf16 range well away from underflow, undo after squaring
        scale = fr.abs().amax(dim=(1, 2), keepdim=True).clamp_min(1e-8)   # [b, 1, 1]
        f = (fr / scale).reshape(b * T, N_FFT)
        f_hi = f.to(torch.bfloat16)
        f_lo = (f - f_hi.float()).to(torch.bfloat16)
        spec = linear(torch.cat([f_hi, f_hi, f_lo], 1).contiguous(), self.basis, out_dtype=torch.float32)
        re, im = spec[:, :201], spec[:, 201:402]
        p = torch.zeros(b * T, 208, dtype=torch.float32, device=self.device)
        p[:, :201] = (re * re + im * im).view(b, T, 201).mul_(scale * scale).view(b * T, 201)
        pmax = p.view(b, T, 208).amax(dim=(1, 2), keepdim=True).clamp_min(1e-20)   # [b, 1, 1]
        mel = linear((p.view(b, T, 208) / pmax).view(b * T, 208).to(torch.bfloat16), self.fb,
                     out_dtype=torch.float32).view(b, T, -1) * pmax               # [b, T, n_mels]
        log_spec = torch.clamp(mel, min=1e-10).log10()
        log_spec = torch.maximum(log_spec, log_spec.amax(dim=(1, 2), keepdim=True) - 8.0)
        return ((log_spec + 4.0) / 4.0).transpose(1, 2)
