"""SVA artifact bundles: the reference's on-disk format, loaded and validated.

The format is the reference's (asystemoffields/sva, sva/artifacts.py): a directory holding
``sva_config.json`` (manifest, ``schema_version`` 1) and ``sva_artifacts.pt`` (a torch payload
``{"schema_version": 1, "tensors": {"layers.{i}.q_proj": [H, D, R], "layers.{i}.k_proj": ...,
"layers.{i}.logit_scale": [H], "layers.{i}.coarse_codebooks": [H, S, C, R/S]}, "layer_meta":
{...}}``).  Bundles exported for the reference load unchanged here, and the same validation
errors are raised (sva/artifacts.py:131-167).
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch

SCHEMA_VERSION = 1
WEIGHTS_NAME = "sva_artifacts.pt"
MANIFEST_NAME = "sva_config.json"


@dataclass(frozen=True)
class SVALayerArtifacts:
    """Frozen per-layer tensors of the SVA lookup path (reference sva/artifacts.py:17-27)."""

    q_proj: torch.Tensor
    k_proj: torch.Tensor
    logit_scale: torch.Tensor
    coarse_codebooks: torch.Tensor
    train_loss: float
    hard_loss: float
    route_source: str = "qk"


@dataclass(frozen=True)
class SVAArtifactBundle:
    """Manifest plus per-layer artifacts (reference sva/artifacts.py:30-81)."""

    manifest: dict[str, Any]
    layers: dict[int, SVALayerArtifacts]

    @property
    def model_id(self) -> str | None:
        value = self.manifest.get("model_id")
        return None if value is None else str(value)

    @property
    def rank_dim(self) -> int:
        return int(self.manifest["rank_dim"])

    @property
    def default_shortlist(self) -> int:
        return int(self.manifest.get("default_shortlist", 2048))

    @property
    def default_budget(self) -> int:
        return int(self.manifest.get("default_budget", 512))

    @property
    def coarse_subspaces(self) -> int:
        return int(self.manifest["coarse_subspaces"])

    @property
    def coarse_codewords(self) -> int:
        return int(self.manifest["coarse_codewords"])

    @property
    def layer_count(self) -> int:
        return int(self.manifest.get("layer_count", len(self.layers)))

    def to(self, device: torch.device | str, dtype: torch.dtype | None = None) -> "SVAArtifactBundle":
        """Copy with tensors moved to ``device`` (and ``dtype``, logit scales stay fp32)."""
        moved = {}
        for idx, layer in self.layers.items():
            dt = dtype if dtype is not None else layer.q_proj.dtype
            moved[idx] = SVALayerArtifacts(
                q_proj=layer.q_proj.to(device=device, dtype=dt),
                k_proj=layer.k_proj.to(device=device, dtype=dt),
                logit_scale=layer.logit_scale.to(device=device, dtype=torch.float32),
                coarse_codebooks=layer.coarse_codebooks.to(device=device, dtype=dt),
                train_loss=layer.train_loss,
                hard_loss=layer.hard_loss,
                route_source=layer.route_source,
            )
        return SVAArtifactBundle(dict(self.manifest), moved)


def load_sva_artifact_bundle(artifact_dir: str | Path, map_location: str | torch.device = "cpu") -> SVAArtifactBundle:
    """Load and validate a bundle directory (reference sva/artifacts.py:91-128)."""
    path = Path(artifact_dir)
    with (path / MANIFEST_NAME).open("r", encoding="utf-8") as fh:
        manifest = json.load(fh)
    if int(manifest.get("schema_version", -1)) != SCHEMA_VERSION:
        raise ValueError(f"Unsupported SVA artifact schema: {manifest.get('schema_version')!r}")
    weights = path / manifest.get("weights_file", WEIGHTS_NAME)
    try:
        payload = torch.load(weights, map_location=map_location, weights_only=True)
    except TypeError:  # torch without weights_only
        payload = torch.load(weights, map_location=map_location)
    if int(payload.get("schema_version", -1)) != SCHEMA_VERSION:
        raise ValueError(f"Unsupported SVA weights schema: {payload.get('schema_version')!r}")
    tensors = payload["tensors"]
    layer_meta = payload.get("layer_meta", {})
    layers: dict[int, SVALayerArtifacts] = {}
    for raw in manifest["layers"]:
        idx = int(raw)
        prefix = f"layers.{idx}"
        meta = layer_meta.get(str(idx), {})
        layers[idx] = SVALayerArtifacts(
            q_proj=tensors[f"{prefix}.q_proj"],
            k_proj=tensors[f"{prefix}.k_proj"],
            logit_scale=tensors[f"{prefix}.logit_scale"],
            coarse_codebooks=tensors[f"{prefix}.coarse_codebooks"],
            train_loss=float(meta["train_loss"]) if meta.get("train_loss") is not None else float("nan"),
            hard_loss=float(meta["hard_loss"]) if meta.get("hard_loss") is not None else float("nan"),
            route_source=str(meta.get("route_source", manifest.get("route_source", "qk"))),
        )
    bundle = SVAArtifactBundle(manifest, layers)
    validate_artifact_bundle(bundle)
    return bundle


def save_sva_artifact_bundle(bundle: SVAArtifactBundle, artifact_dir: str | Path) -> Path:
    """Write a bundle in the reference format (manifest + torch payload)."""
    path = Path(artifact_dir)
    path.mkdir(parents=True, exist_ok=True)
    manifest = dict(bundle.manifest)
    manifest.setdefault("schema_version", SCHEMA_VERSION)
    manifest.setdefault("layers", sorted(bundle.layers))
    tensors, meta = {}, {}
    for idx, layer in bundle.layers.items():
        for name in ("q_proj", "k_proj", "logit_scale", "coarse_codebooks"):
            tensors[f"layers.{idx}.{name}"] = getattr(layer, name).detach().cpu()
        meta[str(idx)] = {"train_loss": layer.train_loss, "hard_loss": layer.hard_loss,
                          "route_source": layer.route_source}
    torch.save({"schema_version": SCHEMA_VERSION, "tensors": tensors, "layer_meta": meta},
               path / manifest.get("weights_file", WEIGHTS_NAME))
    with (path / MANIFEST_NAME).open("w", encoding="utf-8") as fh:
        json.dump(manifest, fh, indent=2, sort_keys=True)
    return path


def validate_artifact_bundle(bundle: SVAArtifactBundle) -> None:
    """Manifest / tensor consistency checks (reference sva/artifacts.py:131-167)."""
    if not bundle.layers:
        raise ValueError("SVA artifact bundle contains no layers.")
    rank_dim = bundle.rank_dim
    subspaces = bundle.coarse_subspaces
    codewords = bundle.coarse_codewords
    if rank_dim <= 0:
        raise ValueError(f"rank_dim must be positive, got {rank_dim}.")
    if subspaces <= 0 or rank_dim % subspaces != 0:
        raise ValueError(f"rank_dim={rank_dim} must be divisible by coarse_subspaces={subspaces}.")
    if codewords <= 0:
        raise ValueError(f"coarse_codewords must be positive, got {codewords}.")
    for idx, layer in bundle.layers.items():
        if layer.q_proj.shape != layer.k_proj.shape:
            raise ValueError(f"Layer {idx} q_proj/k_proj shape mismatch: {layer.q_proj.shape} vs {layer.k_proj.shape}.")
        if layer.q_proj.ndim != 3:
            raise ValueError(f"Layer {idx} q_proj must have shape [heads, head_dim, rank_dim].")
        if int(layer.q_proj.shape[-1]) != rank_dim:
            raise ValueError(f"Layer {idx} rank_dim mismatch: {layer.q_proj.shape[-1]} vs {rank_dim}.")
        if layer.logit_scale.ndim != 1 or int(layer.logit_scale.shape[0]) != int(layer.q_proj.shape[0]):
            raise ValueError(f"Layer {idx} logit_scale must have one value per attention head.")
        expected = (int(layer.q_proj.shape[0]), subspaces, codewords, rank_dim // subspaces)
        if tuple(layer.coarse_codebooks.shape) != expected:
            raise ValueError(f"Layer {idx} coarse_codebooks shape mismatch: {tuple(layer.coarse_codebooks.shape)} "
                             f"vs {expected}.")
        if layer.route_source != "qk":
            raise ValueError(f"Layer {idx} uses route_source={layer.route_source!r}. "
                             "The production adapter currently supports qk artifacts.")
