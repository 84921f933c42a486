"""Multimodal hooks and encoder contracts (reference ``core/multimodal/*``, 674 LoC).

* ``ModalityProjector``: SwiGLU MLP (encoder dim -> D) + RMSNorm; when disabled it
  holds one frozen ``_disabled`` parameter so checkpoints keep the same key.
* ``ResidualSideChannel``: ``h + alpha * mem(h)`` (alpha = 0, no memory by default).
* ``GenerationHeadHook``: zero-init D -> VQ-slot linear, frozen unless enabled.
* Vision: ``VisionEncoderConfig``, ``deepstack_fuse`` (concat of layers -1/-5/-9),
  ``FakeViT`` (hermetic stand-in), ``SigLIP2Wrapper`` (lazy HF load), ``VisionTokenizer``.
* Audio: ``AudioEncoderConfig`` (12.5 Hz output), ``FakeWhisperEncoder`` (2x pool),
  ``WhisperLargeV3Wrapper`` (lazy HF), ``AudioTokenizer`` (4-frame fuse MLP).
* Video: ``VideoTokenizer`` protocol, ``FakeVideoTokenizer``, ``encode_video_clips``.
* Reasoning effort: ``EffortConfig``, ``EffortRouter`` (zero-init budget/terminate
  heads) and the tier helpers.
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import Protocol

import torch
import torch.nn.functional as F
from pydantic import BaseModel, ConfigDict
from torch import Tensor, nn

from saint_llm_b200.models.attention.common import RMSNorm


class ModalityProjector(nn.Module):
    def __init__(self, in_dim: int, hidden_dim: int, enabled: bool = False) -> None:
        super().__init__()
        self.enabled = enabled
        if enabled:
            self.up = nn.Linear(in_dim, hidden_dim, bias=False)
            self.gate = nn.Linear(in_dim, hidden_dim, bias=False)
            self.down = nn.Linear(hidden_dim, hidden_dim, bias=False)
            self.out_norm = RMSNorm(hidden_dim)
        else:
            self.register_parameter("_disabled", nn.Parameter(torch.zeros(1), requires_grad=False))

    def forward(self, x: Tensor) -> Tensor:
        if not self.enabled:
            raise RuntimeError("ModalityProjector is disabled")
        return self.out_norm(self.down(F.silu(self.gate(x)) * self.up(x)))


class ResidualSideChannel(nn.Module):
    def __init__(self, hidden_dim: int, alpha_init: float = 0.0) -> None:
        super().__init__()
        self.hidden_dim = hidden_dim
        self.alpha = nn.Parameter(torch.full((1,), float(alpha_init)))
        self._mem_module: nn.Module | None = None

    def attach(self, mem_module: nn.Module) -> None:
        self._mem_module = mem_module

    @property
    def active(self) -> bool:
        # Host-side check (no device sync): a memory module must be attached.
        return self._mem_module is not None

    def forward(self, h: Tensor) -> Tensor:
        if self._mem_module is None:
            return h
        return h + self.alpha * self._mem_module(h)


class GenerationHeadHook(nn.Module):
    def __init__(self, hidden_dim: int, vocab_slots: int, enabled: bool = False) -> None:
        super().__init__()
        self.enabled = enabled
        self.proj = nn.Linear(hidden_dim, vocab_slots, bias=False)
        nn.init.zeros_(self.proj.weight)
        if not enabled:
            self.proj.weight.requires_grad_(False)

    def forward(self, h: Tensor) -> Tensor:
        return self.proj(h)


# ---------------------------------------------------------------------------------- vision
class VisionEncoderConfig(BaseModel):
    model_config = ConfigDict(frozen=True, extra="forbid")
    encoder_name: str = "google/siglip2-so400m-patch14-384"
    encoder_hidden_dim: int = 1152
    deepstack_layers: tuple[int, ...] = (-1, -5, -9)
    deepstack_enabled: bool = True
    freeze: bool = True
    image_size: int = 384
    patch_size: int = 14
    adaptive_token_min: int = 64
    adaptive_token_max: int = 1280

    @property
    def output_dim(self) -> int:
        return self.encoder_hidden_dim * (len(self.deepstack_layers) if self.deepstack_enabled else 1)


def deepstack_fuse(hidden_states: Sequence[Tensor], layers: tuple[int, ...]) -> Tensor:
    return torch.cat([hidden_states[i] for i in layers], dim=-1)


class FakeViT(nn.Module):
    """Hermetic ViT stand-in: patch conv + per-layer additive offsets."""

    def __init__(self, cfg: VisionEncoderConfig, n_layers: int = 12) -> None:
        super().__init__()
        self.cfg = cfg
        self.n_layers = n_layers
        self.patch_proj = nn.Conv2d(3, cfg.encoder_hidden_dim, kernel_size=cfg.patch_size,
                                    stride=cfg.patch_size)
        self.layer_perturbations = nn.ParameterList(
            nn.Parameter(torch.randn(cfg.encoder_hidden_dim) * 0.01) for _ in range(n_layers)
        )

    def forward(self, pixel_values: Tensor) -> dict[str, Tensor | list[Tensor]]:
        x = self.patch_proj(pixel_values).flatten(2).transpose(1, 2)
        states = [x]
        for off in self.layer_perturbations:
            x = x + off.view(1, 1, -1)
            states.append(x)
        return {"last_hidden_state": states[-1], "hidden_states": states,
                "n_patches": torch.tensor(states[0].shape[1])}


class SigLIP2Wrapper(nn.Module):
    """SigLIP-2 vision tower, loaded lazily from a local HF checkpoint on first use."""

    def __init__(self, cfg: VisionEncoderConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self._encoder: nn.Module | None = None

    def _load(self) -> nn.Module:
        if self._encoder is None:
            from transformers import AutoModel

            enc = AutoModel.from_pretrained(self.cfg.encoder_name)
            enc = getattr(enc, "vision_model", enc)
            if self.cfg.freeze:
                enc.requires_grad_(False)
                enc.eval()
            self._encoder = enc
        return self._encoder

    def forward(self, pixel_values: Tensor) -> dict[str, Tensor | list[Tensor]]:
        out = self._load()(pixel_values, output_hidden_states=True)
        return {"last_hidden_state": out.last_hidden_state, "hidden_states": list(out.hidden_states)}


class VisionTokenizer(nn.Module):
    def __init__(self, cfg: VisionEncoderConfig, encoder: nn.Module) -> None:
        super().__init__()
        self.cfg = cfg
        self.encoder = encoder

    def forward(self, pixel_values: Tensor) -> Tensor:
        out = self.encoder(pixel_values)
        if self.cfg.deepstack_enabled:
            return deepstack_fuse(out["hidden_states"], self.cfg.deepstack_layers)
        return out["last_hidden_state"]


# ----------------------------------------------------------------------------------- audio
class AudioEncoderConfig(BaseModel):
    model_config = ConfigDict(frozen=True, extra="forbid")
    encoder_name: str = "openai/whisper-large-v3"
    encoder_hidden_dim: int = 1280
    n_mel_bins: int = 128
    sample_rate: int = 16000
    chunk_duration_sec: int = 30
    downsample_factor: int = 4
    freeze: bool = True

    @property
    def output_dim(self) -> int:
        return self.encoder_hidden_dim

    @property
    def output_rate_hz(self) -> float:
        return 100.0 / (2 * self.downsample_factor)


class FakeWhisperEncoder(nn.Module):
    def __init__(self, cfg: AudioEncoderConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.proj = nn.Conv1d(cfg.n_mel_bins, cfg.encoder_hidden_dim, kernel_size=3, stride=2, padding=1)

    def forward(self, mel: Tensor) -> Tensor:
        return self.proj(mel).transpose(1, 2).contiguous()


class WhisperLargeV3Wrapper(nn.Module):
    def __init__(self, cfg: AudioEncoderConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self._encoder: nn.Module | None = None

    def _load(self) -> nn.Module:
        if self._encoder is None:
            from transformers import WhisperModel

            enc = WhisperModel.from_pretrained(self.cfg.encoder_name).encoder
            if self.cfg.freeze:
                enc.requires_grad_(False)
                enc.eval()
            self._encoder = enc
        return self._encoder

    def forward(self, mel: Tensor) -> Tensor:
        return self._load()(mel).last_hidden_state


class AudioTokenizer(nn.Module):
    def __init__(self, cfg: AudioEncoderConfig, encoder: nn.Module) -> None:
        super().__init__()
        self.cfg = cfg
        self.encoder = encoder
        f, d = cfg.downsample_factor, cfg.encoder_hidden_dim
        self.downsample: nn.Module = (
            nn.Sequential(nn.Linear(d * f, d, bias=False), nn.GELU(), nn.Linear(d, d, bias=False))
            if f > 1 else nn.Identity()
        )

    def forward(self, mel: Tensor) -> Tensor:
        enc = self.encoder(mel)
        f = self.cfg.downsample_factor
        if f <= 1:
            return enc
        b, t, d = enc.shape
        pad = (-t) % f
        if pad:
            enc = F.pad(enc, (0, 0, 0, pad))
        return self.downsample(enc.reshape(b, (t + pad) // f, f * d))


# ----------------------------------------------------------------------------------- video
class VideoTokenizer(Protocol):
    @property
    def vision_dim(self) -> int: ...

    @property
    def patches_per_frame(self) -> int: ...

    def encode(self, video: Tensor) -> Tensor: ...


class FakeVideoTokenizer(nn.Module):
    """Deterministic (T,3,H,W) -> (T*P, dim): mean colour per frame through a fixed projection."""

    def __init__(self, *, vision_dim: int, patches_per_frame: int, seed: int = 0) -> None:
        super().__init__()
        if vision_dim <= 0 or patches_per_frame <= 0:
            raise ValueError("vision_dim and patches_per_frame must be positive")
        self._vision_dim = vision_dim
        self._patches_per_frame = patches_per_frame
        gen = torch.Generator().manual_seed(seed)
        self.register_buffer("projection", torch.randn(3, vision_dim, generator=gen), persistent=False)

    @property
    def vision_dim(self) -> int:
        return self._vision_dim

    @property
    def patches_per_frame(self) -> int:
        return self._patches_per_frame

    def encode(self, video: Tensor) -> Tensor:
        if video.dim() != 4 or video.shape[1] != 3:
            raise ValueError(f"video must be (T, 3, H, W); got {tuple(video.shape)}")
        t = video.shape[0]
        feat = video.float().mean(dim=(-2, -1)) @ self.projection
        offs = torch.arange(self._patches_per_frame, device=video.device, dtype=feat.dtype)[:, None] * 1e-3
        return (feat[:, None, :] + offs[None]).reshape(t * self._patches_per_frame, self._vision_dim)


def encode_video_clips(clips: list[Tensor], tokenizer: VideoTokenizer) -> list[Tensor]:
    return [tokenizer.encode(c) for c in clips]


# ------------------------------------------------------------------------- reasoning effort
class EffortConfig(BaseModel):
    model_config = ConfigDict(frozen=True, extra="forbid")
    n_tiers: int = 5
    hidden: int = 64
    enabled: bool = False


class EffortRouter(nn.Module):
    """Zero-initialised budget / terminate heads conditioned on a pooled query + tier."""

    def __init__(self, hidden_dim: int, cfg: EffortConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.tier_emb = nn.Embedding(cfg.n_tiers, cfg.hidden)
        self.fuse = nn.Linear(hidden_dim + cfg.hidden, cfg.hidden, bias=True)
        self.budget_head = nn.Linear(cfg.hidden, 1, bias=True)
        self.terminate_head = nn.Linear(cfg.hidden, 1, bias=True)
        for p in self.parameters():
            nn.init.zeros_(p)

    def forward(self, query_pooled: Tensor, effort_tier: Tensor) -> dict[str, Tensor]:
        if effort_tier.dim() != 1:
            raise ValueError("effort_tier must be 1D (B,)")
        if bool(((effort_tier < 0) | (effort_tier >= self.cfg.n_tiers)).any()):
            raise ValueError(f"effort_tier values must be in [0, {self.cfg.n_tiers})")
        z = torch.relu(self.fuse(torch.cat([query_pooled, self.tier_emb(effort_tier)], dim=-1)))
        return {"budget": torch.relu(self.budget_head(z).squeeze(-1)),
                "terminate_logit": self.terminate_head(z).squeeze(-1)}


EFFORT_TIER_NAMES: tuple[str, ...] = ("low", "medium", "high", "xhigh", "max")


def effort_tier_to_id(name: str) -> int:
    key = name.lower()
    if key not in EFFORT_TIER_NAMES:
        raise ValueError(f"unknown effort tier {name!r}")
    return EFFORT_TIER_NAMES.index(key)


def effort_id_to_token(tier_id: int) -> str:
    if not 0 <= tier_id < len(EFFORT_TIER_NAMES):
        raise ValueError(f"tier_id {tier_id} out of range")
    return f"<|effort:{tier_id}|>"


__all__ = [
    "EFFORT_TIER_NAMES",
    "AudioEncoderConfig",
    "AudioTokenizer",
    "EffortConfig",
    "EffortRouter",
    "FakeViT",
    "FakeVideoTokenizer",
    "FakeWhisperEncoder",
    "GenerationHeadHook",
    "ModalityProjector",
    "ResidualSideChannel",
    "SigLIP2Wrapper",
    "VideoTokenizer",
    "VisionEncoderConfig",
    "VisionTokenizer",
    "WhisperLargeV3Wrapper",
    "deepstack_fuse",
    "effort_id_to_token",
    "effort_tier_to_id",
    "encode_video_clips",
]
