"""YAML model configs and the ``get_model_from_config`` entry point.

Mirrors the pymss-core calls the reference makes
(``get_model_from_config(model_type, config_path, model_kwargs_override=...)``
and ``load_config(path)``, src/pymsst/training/module.py:9, 76, 330-336):
the returned config supports attribute and ``.get`` access, and the model
kwargs are ``config.model`` plus the override.  Mel-band RoFormer configs
without ``mlp_hidden_layers`` keep the legacy meaning of
``mask_estimator_depth`` (that many hidden layers), as the reference's
``_model_kwargs_override`` arranges.
"""
from __future__ import annotations

from pathlib import Path
from typing import Any

import yaml

from .roformer import BSRoformer, MelBandRoformer

MODEL_TYPES = {"bs_roformer": BSRoformer, "mel_band_roformer": MelBandRoformer}


class ConfigDict(dict):
    """dict with attribute access, recursively."""

    def __init__(self, data: dict | None = None):
        super().__init__()
        for key, value in (data or {}).items():
            self[key] = value

    def __setitem__(self, key, value):
        super().__setitem__(key, _wrap(value))

    def __getattr__(self, key):
        try:
            return self[key]
        except KeyError as exc:
            raise AttributeError(key) from exc

    def __setattr__(self, key, value):
        self[key] = value

    def to_plain(self) -> dict:
        return {k: (v.to_plain() if isinstance(v, ConfigDict) else v) for k, v in self.items()}


def _wrap(value: Any) -> Any:
    if isinstance(value, dict) and not isinstance(value, ConfigDict):
        return ConfigDict(value)
    if isinstance(value, list):
        return [_wrap(v) for v in value]
    return value


def load_config(path: str | Path) -> ConfigDict:
    with open(path, encoding="utf-8") as handle:
        return ConfigDict(yaml.safe_load(handle) or {})


def model_kwargs(model_type: str, config: ConfigDict, override: dict | None = None) -> dict:
    kwargs = dict(config.model.to_plain() if isinstance(config.model, ConfigDict) else config.model)
    kwargs.update(override or {})
    if model_type == "mel_band_roformer" and "mlp_hidden_layers" not in kwargs:
        kwargs["mlp_hidden_layers"] = int(kwargs.get("mask_estimator_depth", 1))
    for key in ("freqs_per_bands", "multi_stft_resolutions_window_sizes"):
        if key in kwargs and isinstance(kwargs[key], list):
            kwargs[key] = tuple(kwargs[key])
    return kwargs


def build_model(model_type: str, **kwargs):
    try:
        cls = MODEL_TYPES[model_type]
    except KeyError as exc:
        raise ValueError("model_type must be 'bs_roformer' or 'mel_band_roformer'") from exc
    return cls(**kwargs)


def get_model_from_config(model_type: str, config_path: str | Path, model_kwargs_override: dict | None = None):
    """(model, config) for a pymss-core / MSST YAML config."""
    config = load_config(config_path)
    model = build_model(model_type, **model_kwargs(model_type, config, model_kwargs_override))
    return model, config
