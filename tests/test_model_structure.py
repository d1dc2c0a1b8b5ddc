"""Model structure (CPU): the product modules keep the oracle's (pymss-core's)
constructor arguments and state-dict layout, configs load from YAML, and the
product refuses to run on the CPU."""
from __future__ import annotations

import pytest
import torch
import yaml

from oracle import roformer_ref
from pymsst_b200 import config as cfg
from pymsst_b200 import roformer, synthetic
from pymsst_b200._native import FusedKernelUnavailable
from tests.model_configs import CONFIG0_BSR, CONFIG1_MBR, TINY_BSR, TINY_MBR

CASES = [("bs_roformer", TINY_BSR), ("mel_band_roformer", TINY_MBR), ("bs_roformer", CONFIG0_BSR),
         ("mel_band_roformer", CONFIG1_MBR)]


def _pair(model_type, kwargs):
    ours = cfg.build_model(model_type, **kwargs)
    ref = roformer_ref.build(model_type, **kwargs)
    return ours, ref


@pytest.mark.parametrize("model_type,kwargs", CASES)
def test_state_dict_layout_matches_oracle(model_type, kwargs):
    ours, ref = _pair(model_type, kwargs)
    a, b = ours.state_dict(), ref.state_dict()
    assert list(a.keys()) == list(b.keys())
    for k in a:
        assert a[k].shape == b[k].shape, k
    ours.load_state_dict(b, strict=True)
    assert sum(p.numel() for p in ours.parameters()) == sum(p.numel() for p in ref.parameters())


def test_config0_parameter_count_and_bands():
    ours, _ = _pair("bs_roformer", CONFIG0_BSR)
    n = sum(p.numel() for p in ours.parameters())
    assert 24e6 < n < 25e6
    assert len(ours.band_split.dim_inputs) == 62 and sum(ours.band_split.dim_inputs) == 4100
    mbr, _ = _pair("mel_band_roformer", CONFIG1_MBR)
    assert len(mbr.band_split.dim_inputs) == 60 and sum(mbr.band_split.dim_inputs) == 1979 * 4


def test_mel_legacy_mask_depth_layers():
    """mask_estimator_depth=2 without mlp_hidden_layers -> 3 linear layers (module.py:330-336)."""
    kwargs = dict(TINY_MBR, mask_estimator_depth=2)
    model = cfg.build_model("mel_band_roformer", **cfg.model_kwargs("mel_band_roformer", cfg.ConfigDict({"model": kwargs})))
    mlp = model.mask_estimators[0].to_freqs[0][0]
    assert len([m for m in mlp if isinstance(m, torch.nn.Linear)]) == 3
    model = cfg.build_model("mel_band_roformer", **dict(kwargs, mlp_hidden_layers=1))
    assert len([m for m in model.mask_estimators[0].to_freqs[0][0] if isinstance(m, torch.nn.Linear)]) == 2


def test_get_model_from_config_yaml(tmp_path):
    path = tmp_path / "bsr.yaml"
    path.write_text(yaml.safe_dump({"model": dict(TINY_BSR, freqs_per_bands=list(TINY_BSR["freqs_per_bands"])),
                                    "training": {"lr": 1e-4}}))
    model, config = cfg.get_model_from_config("bs_roformer", path)
    assert isinstance(model, roformer.BSRoformer)
    assert config.training.lr == 1e-4 and config.training.get("q", 0.95) == 0.95
    with pytest.raises(ValueError, match="model_type"):
        cfg.build_model("htdemucs")


def test_forward_on_cpu_fails_loudly():
    model = cfg.build_model("bs_roformer", **TINY_BSR)
    with pytest.raises(FusedKernelUnavailable):
        model(torch.randn(1, 2, 256))


def test_synthetic_generator_is_seeded():
    a = synthetic.make_batch(2, 4096, seed=3)
    b = synthetic.make_batch(2, 4096, seed=3)
    c = synthetic.make_batch(2, 4096, seed=4)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert not torch.equal(a[0], c[0])
    mix, tgt = a
    assert mix.shape == tgt.shape == (2, 2, 4096)
    noise = synthetic.pink_noise(44100, 2, torch.Generator().manual_seed(0))
    assert abs(float(noise.pow(2).mean().sqrt()) - 0.1) < 1e-6
    mix4, tgt4 = synthetic.make_batch(1, 1024, seed=0, stems=4)
    assert tgt4.shape == (1, 4, 2, 1024)
    torch.testing.assert_close(mix4, tgt4.sum(1))


@pytest.mark.parametrize("model_type,kwargs", [("bs_roformer", TINY_BSR), ("mel_band_roformer", TINY_MBR)])
def test_checkpoint_package_round_trip(tmp_path, model_type, kwargs):
    """The reference's export package (src/pymsst/export/checkpoint.py:10-31): written from this package's model,
    loaded back (model rebuilt from the package's config) and into the oracle (pymss-core's layout), and one
    written from the oracle's model loaded here; every tensor survives bit for bit."""
    from pymsst_b200.checkpoint import export_core_checkpoint, load_core_checkpoint

    torch.manual_seed(3)
    ours, ref = _pair(model_type, kwargs)
    conf = {"model": dict(kwargs), "training": {"batch_size": 2}}
    path = export_core_checkpoint(ours, tmp_path / "ours.ckpt", model_type=model_type, config=conf,
                                  metadata={"epoch": 1})
    package = torch.load(path, map_location="cpu", weights_only=True)
    assert set(package) == {"state_dict", "model_type", "config", "metadata"}
    assert package["model_type"] == model_type and package["metadata"] == {"epoch": 1}
    assert all(t.device.type == "cpu" for t in package["state_dict"].values())
    back, _ = load_core_checkpoint(path)
    ref.load_state_dict(package["state_dict"], strict=True)
    want = ours.state_dict()
    for k, v in back.state_dict().items():
        assert torch.equal(v, want[k]), k
    for k, v in ref.state_dict().items():
        assert torch.equal(v, want[k]), k
    # the other direction: the oracle's weights exported in the same layout load into this package's model
    torch.manual_seed(4)
    _, ref2 = _pair(model_type, kwargs)
    path2 = export_core_checkpoint(ref2, tmp_path / "ref.ckpt", model_type=model_type)
    mine, _ = load_core_checkpoint(path2, model=cfg.build_model(model_type, **kwargs))
    for k, v in ref2.state_dict().items():
        assert torch.equal(mine.state_dict()[k], v), k
    with pytest.raises(ValueError, match="no config"):
        load_core_checkpoint(path2)
