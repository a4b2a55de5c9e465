"""Refine-stage weights from safetensors (refine_stage.load_params, the
reference's Refiner::load_file, src/dsine_refine.cpp:185-194): names and
shapes, F32 / F16 / BF16 widening, extra tensors ignored, errors for a
missing tensor or a wrong shape. Fixtures are written with the safetensors
library, which cross-checks the reader."""
import pytest
import torch

safetensors_torch = pytest.importorskip("safetensors.torch")


def write(path, tensors):
    safetensors_torch.save_file({k: v.contiguous() for k, v in tensors.items()}, str(path))


def test_load_params_round_trip(tmp_path):
    from brovisionml_b200.refine_stage import load_params, param_shapes, random_params

    p = random_params("cpu", seed=3)
    dts = [torch.float32, torch.float16, torch.bfloat16]
    stored = {k: v.to(dts[i % 3]) for i, (k, v) in enumerate(sorted(p.items()))}
    stored["encoder.stem.weight"] = torch.zeros(3, 3)  # other parts of the model file
    write(tmp_path / "model.safetensors", stored)
    got = load_params(str(tmp_path / "model.safetensors"))
    assert set(got) == set(param_shapes())
    for k, v in got.items():
        assert v.dtype == torch.float32 and tuple(v.shape) == param_shapes()[k]
        assert torch.equal(v, stored[k].float()), k
    # the reference's layout: 3 GRU convs + 4 heads x 3 convs, weight and bias
    assert len(got) == 2 * (3 + 4 * 3)


def test_load_params_errors(tmp_path):
    from brovisionml_b200.refine_stage import load_params, random_params

    p = random_params("cpu", seed=1)
    q = dict(p)
    del q["xy_head.4.bias"]
    write(tmp_path / "a.safetensors", q)
    with pytest.raises(RuntimeError, match="missing tensor 'xy_head.4.bias'"):
        load_params(str(tmp_path / "a.safetensors"))
    q = dict(p)
    q["gru.convq.weight"] = torch.zeros(64, 130, 3, 3)
    write(tmp_path / "b.safetensors", q)
    with pytest.raises(RuntimeError, match="gru.convq.weight' has shape"):
        load_params(str(tmp_path / "b.safetensors"))
    (tmp_path / "c.safetensors").write_bytes(b"\xff" * 16)
    with pytest.raises(RuntimeError, match="not a safetensors file"):
        load_params(str(tmp_path / "c.safetensors"))
