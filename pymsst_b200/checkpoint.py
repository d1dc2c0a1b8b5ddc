"""Checkpoint packages in the reference's export format.

The reference exports a trained model as one ``torch.save`` package
(src/pymsst/export/checkpoint.py:10-31): ``{"state_dict": {key: CPU tensor},
"model_type": str}`` plus ``"config"`` (the config as plain data, pymss-core's
``to_plain``) and ``"metadata"`` when given.  The models here keep pymss-core's
state-dict keys, so such a package loads into them strictly, and a package
written here loads into pymss-core: ``export_core_checkpoint`` writes the same
layout, ``load_core_checkpoint`` reads one (building the model from the
package's config when no model is given).
"""
from __future__ import annotations

from pathlib import Path
from typing import Any

import torch

from . import config as cfg


def _plain(value: Any) -> Any:
    if isinstance(value, cfg.ConfigDict):
        return value.to_plain()
    if isinstance(value, dict):
        return {k: _plain(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [_plain(v) for v in value]
    return value


def _unwrap(model: torch.nn.Module) -> torch.nn.Module:
    return model.module if hasattr(model, "module") else model


def export_core_checkpoint(model: torch.nn.Module, path: str | Path, *, model_type: str, config: Any | None = None,
                           metadata: dict[str, Any] | None = None) -> Path:
    """Write ``model`` (unwrapped from DDP) as the reference's export package; returns the path."""
    output_path = Path(path)
    output_path.parent.mkdir(parents=True, exist_ok=True)
    state = _unwrap(model).state_dict()
    package: dict[str, Any] = {
        "state_dict": {key: value.detach().cpu() for key, value in state.items()},
        "model_type": model_type,
    }
    if config is not None:
        package["config"] = _plain(config)
    if metadata:
        package["metadata"] = metadata
    torch.save(package, output_path)
    return output_path


def load_core_checkpoint(path: str | Path, model: torch.nn.Module | None = None,
                         model_kwargs_override: dict | None = None) -> tuple[torch.nn.Module, dict]:
    """(model, package) from an export package: the state dict loaded strictly into ``model``, or into a model
    built from the package's ``model_type`` and ``config`` (its ``model`` section plus the override)."""
    package = torch.load(Path(path), map_location="cpu", weights_only=True)
    if not isinstance(package, dict) or "state_dict" not in package or "model_type" not in package:
        raise ValueError(f"{path}: not a checkpoint package (needs 'state_dict' and 'model_type')")
    if model is None:
        if "config" not in package:
            raise ValueError(f"{path}: the package has no config to build the model from; pass a model")
        conf = cfg.ConfigDict(package["config"])
        model = cfg.build_model(package["model_type"],
                                **cfg.model_kwargs(package["model_type"], conf, model_kwargs_override))
    _unwrap(model).load_state_dict(package["state_dict"], strict=True)
    return model, package
