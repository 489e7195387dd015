"""The safetensors loader (qmoe_b200.loader, qmoe-rs src/loader.rs:204-359):
key layout, shapes, missing-tensor errors, the uniform router of a layer
without one, shared / flattened layers.  The file is written with the
reference's key names from the committed moe_tiny fixture, whose bytes
quantize.py produced; the GPU test runs the loaded layer against one built
from the same arrays."""
import os

import numpy as np
import pytest
import torch
from safetensors.torch import save_file

from qmoe_b200 import MoEConfig, QMoELayer
from qmoe_b200 import loader

HERE = os.path.dirname(os.path.abspath(__file__))
PROJ = {"gate": "gate_proj", "up": "up_proj", "down": "down_proj"}


def tiny():
    z = np.load(os.path.join(HERE, "golden", "moe_tiny.npz"))
    E, H, I, Is, T = [int(v) for v in z["dims"]]
    return z, E, H, I, Is, T


def packed2d(a, rows):
    return torch.from_numpy(np.ascontiguousarray(a).reshape(rows, -1))


def write_layer(path, layer=3, with_gate=True, with_shared=True, drop=None):
    z, E, H, I, Is, T = tiny()
    pre = f"layers.{layer}.moe"
    d = {}
    if with_gate:
        d[f"{pre}.gate.weight"] = torch.from_numpy(z["gate_w"])
    rows = {"gate": I, "up": I, "down": H}
    for e in range(E):
        for n in ("gate", "up", "down"):
            d[f"{pre}.experts.{e}.{PROJ[n]}.weight"] = packed2d(z[f"e{e}_{n}_packed"], rows[n])
            d[f"{pre}.experts.{e}.{PROJ[n]}.scales"] = torch.from_numpy(z[f"e{e}_{n}_scales"])
    if with_shared:
        srows = {"gate": Is, "up": Is, "down": H}
        for n in ("gate", "up", "down"):
            d[f"{pre}.shared_experts.{PROJ[n]}.weight"] = packed2d(z[f"shared_{n}_packed"], srows[n])
            d[f"{pre}.shared_experts.{PROJ[n]}.scales"] = torch.from_numpy(z[f"shared_{n}_scales"])
    d["layers.0.attn.q_proj.weight"] = torch.zeros(4, 4)          # other tensors are ignored
    if drop:
        del d[drop]
    save_file(d, str(path))
    return z, E, H, I, Is, T


def test_read_layer_maps_the_reference_keys(tmp_path):
    f = tmp_path / "m.safetensors"
    z, E, H, I, Is, T = write_layer(f)
    t = loader.read_layer(str(f), 3, MoEConfig(E, 2, H, I))
    assert not t.flattened and t.config.shared_intermediate_dim == Is
    assert torch.equal(t.gate_weight, torch.from_numpy(z["gate_w"]))
    for e in range(E):
        for j, n in enumerate(("gate", "up", "down")):
            p, s = t.experts[e][j]
            assert np.array_equal(p.numpy().reshape(-1), z[f"e{e}_{n}_packed"].reshape(-1))
            assert np.array_equal(s.numpy(), z[f"e{e}_{n}_scales"])
    for j, n in enumerate(("gate", "up", "down")):
        assert np.array_equal(t.shared[j][0].numpy().reshape(-1), z[f"shared_{n}_packed"].reshape(-1))


def test_read_layer_without_router_or_shared(tmp_path):
    f = tmp_path / "m.safetensors"
    z, E, H, I, Is, T = write_layer(f, with_gate=False, with_shared=False)
    t = loader.read_layer(str(f), 3, MoEConfig(E, 2, H, I, shared_intermediate_dim=Is))
    assert torch.equal(t.gate_weight, torch.ones(E, H))     # src/loader.rs:417-424
    assert t.shared is None and t.config.shared_intermediate_dim == 0


def test_missing_tensor_names_its_key(tmp_path):
    f = tmp_path / "m.safetensors"
    key = "layers.3.moe.experts.2.down_proj.scales"
    z, E, H, I, Is, T = write_layer(f, drop=key)
    with pytest.raises(KeyError, match=key.replace(".", r"\.")):
        loader.read_layer(str(f), 3, MoEConfig(E, 2, H, I))


def test_shape_mismatch_is_rejected(tmp_path):
    f = tmp_path / "m.safetensors"
    z, E, H, I, Is, T = write_layer(f)
    with pytest.raises(ValueError):
        loader.read_layer(str(f), 3, MoEConfig(E, 2, H, 2 * I))     # wrong intermediate_dim


def test_flattened_layer_is_read_as_one_ffn(tmp_path):
    z, E, H, I, Is, T = tiny()
    d = {}
    srows = {"gate": Is, "up": Is, "down": H}
    for n in ("gate", "up", "down"):
        d[f"layers.0.moe.{PROJ[n]}.weight"] = packed2d(z[f"shared_{n}_packed"], srows[n])
        d[f"layers.0.moe.{PROJ[n]}.scales"] = torch.from_numpy(z[f"shared_{n}_scales"])
    f = tmp_path / "flat.safetensors"
    save_file(d, str(f))
    t = loader.read_layer(str(f), 0, MoEConfig(E, 2, H, I))
    assert t.flattened and t.experts == [] and t.config.shared_intermediate_dim == Is
    assert t.shared[0][0].shape == (Is, H // 4)


@pytest.mark.gpu
def test_loaded_layer_matches_direct_construction(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    f = tmp_path / "m.safetensors"
    z, E, H, I, Is, T = write_layer(f)
    cfg = MoEConfig(E, 2, H, I, shared_intermediate_dim=Is)
    np_exp = [[(z[f"e{e}_{n}_packed"].reshape(-1), z[f"e{e}_{n}_scales"])
               for n in ("gate", "up", "down")] for e in range(E)]
    np_sh = [(z[f"shared_{n}_packed"].reshape(-1), z[f"shared_{n}_scales"])
             for n in ("gate", "up", "down")]
    direct = QMoELayer(cfg, z["gate_w"], np_exp, shared=np_sh)
    loaded = loader.load_moe_layer(str(f), 3, MoEConfig(E, 2, H, I))
    a = direct.forward(z["x"])
    b = loaded.forward(z["x"])
    assert np.array_equal(np.asarray(a), np.asarray(b))
    # and the loaded layer against the oracle on the same arrays
    from oracle import oracle as qo
    ref, _, _ = qo.layer_forward(qo.MoEConfig(E, 2, H, I, Is), z["gate_w"], np_exp, z["x"],
                                 shared=np_sh)
    err = float(np.max(np.abs(np.asarray(b) - ref)) / np.max(np.abs(ref)))
    assert err <= 1e-4


@pytest.mark.gpu
def test_loaded_flattened_layer_is_its_ffn(tmp_path):
    # src/loader.rs:452-456: a flattened layer has no routed experts; the
    # block's output is 0 (QMoELayer::forward on empty experts, src/moe.rs:46-48)
    # plus the FFN loaded as the shared expert (src/model.rs:386-389)
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from oracle import oracle as qo
    z, E, H, I, Is, T = tiny()
    d = {}
    srows = {"gate": Is, "up": Is, "down": H}
    for n in ("gate", "up", "down"):
        d[f"layers.0.moe.{PROJ[n]}.weight"] = packed2d(z[f"shared_{n}_packed"], srows[n])
        d[f"layers.0.moe.{PROJ[n]}.scales"] = torch.from_numpy(z[f"shared_{n}_scales"])
    f = tmp_path / "flat.safetensors"
    save_file(d, str(f))
    layer = loader.load_moe_layer(str(f), 0, MoEConfig(E, 2, H, I))
    out, idx, w = layer.forward(z["x"], return_routing=True)
    np_sh = [(z[f"shared_{n}_packed"].reshape(-1), z[f"shared_{n}_scales"])
             for n in ("gate", "up", "down")]
    ref = qo.shared_forward(np_sh, z["x"], H, Is)
    err = float(np.max(np.abs(np.asarray(out) - ref)) / np.max(np.abs(ref)))
    assert err <= 1e-4
    assert np.all(np.asarray(idx) == -1) and np.all(np.asarray(w) == 0.0)
