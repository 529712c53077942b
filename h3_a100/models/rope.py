"""3-D rotary position tables for the joint video/text/audio sequence.

Head dims are split into (t, h, w) groups of rotation pairs.  Video token
``(f, y, x)`` of the latent patch grid rotates by ``(f*w_t, y*w_h, x*w_w)``;
an audio token rotates only in the t group, at its time mapped onto the video
frame axis, so audio and video that play at the same moment share a phase;
text tokens are unrotated.  Frequencies are ``base**(-2i/d_group)``.
Tables are ``cos, sin: [T, head_dim/2]`` in fp32, in the token order
``[video | text | audio]`` used by the DiT.
"""

from __future__ import annotations

import torch


def axis_pairs(head_dim: int) -> tuple[int, int, int]:
    pairs = head_dim // 2
    t = pairs // 4
    h = (pairs - t) // 2
    w = pairs - t - h
    return t, h, w


def _freqs(n_pairs: int, base: float) -> torch.Tensor:
    if n_pairs == 0:
        return torch.zeros(0, dtype=torch.float64)
    return base ** (-torch.arange(n_pairs, dtype=torch.float64) / n_pairs)


def rope_tables(
    grid: tuple[int, int, int],
    n_text: int,
    n_audio: int,
    head_dim: int,
    base: float = 10000.0,
    device: torch.device | str = "cpu",
) -> tuple[torch.Tensor, torch.Tensor]:
    frames, height, width = grid
    pt, ph, pw = axis_pairs(head_dim)
    ft, fh, fw = _freqs(pt, base), _freqs(ph, base), _freqs(pw, base)
    f = torch.arange(frames, dtype=torch.float64)
    y = torch.arange(height, dtype=torch.float64)
    x = torch.arange(width, dtype=torch.float64)
    ang_t = (f[:, None, None, None] * ft).expand(frames, height, width, pt)
    ang_h = (y[None, :, None, None] * fh).expand(frames, height, width, ph)
    ang_w = (x[None, None, :, None] * fw).expand(frames, height, width, pw)
    video = torch.cat([ang_t, ang_h, ang_w], -1).reshape(frames * height * width, pt + ph + pw)
    text = torch.zeros(n_text, pt + ph + pw, dtype=torch.float64)
    if n_audio:
        at = torch.arange(n_audio, dtype=torch.float64) * (frames / max(n_audio, 1))
        audio = torch.cat(
            [at[:, None] * ft, torch.zeros(n_audio, ph + pw, dtype=torch.float64)], -1
        )
    else:
        audio = torch.zeros(0, pt + ph + pw, dtype=torch.float64)
    angles = torch.cat([video, text, audio], 0)
    return angles.cos().float().to(device), angles.sin().float().to(device)
