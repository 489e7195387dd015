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


# ---------------------------------------------------------------------------
# model level: configuration, post-attention LayerNorm, block chains
# ---------------------------------------------------------------------------

def write_model(path, with_norm3=True):
    """Layer 0 flattened (its FFN = the fixture's shared expert), layer 3
    per-expert with a shared expert; layer 3's post_attention_layernorm in the
    file when with_norm3, layer 0's never."""
    z, E, H, I, Is, T = tiny()
    d = {}
    srows = {"gate": Is, "up": Is, "down": H}
    for n in ("gate", "up", "down"):
        d[f"layers.0.moe.{PROJ[n]}.weight"] = packed2d(z[f"shared_{n}_packed"], srows[n])
        d[f"layers.0.moe.{PROJ[n]}.scales"] = torch.from_numpy(z[f"shared_{n}_scales"])
    pre = "layers.3.moe"
    d[f"{pre}.gate.weight"] = torch.from_numpy(z["gate_w"])
    rows = {"gate": I, "up": I, "down": H}
    for e in range(E):
        for n in ("gate", "up", "down"):
            d[f"{pre}.experts.{e}.{PROJ[n]}.weight"] = packed2d(z[f"e{e}_{n}_packed"], rows[n])
            d[f"{pre}.experts.{e}.{PROJ[n]}.scales"] = torch.from_numpy(z[f"e{e}_{n}_scales"])
    for n in ("gate", "up", "down"):
        d[f"{pre}.shared_experts.{PROJ[n]}.weight"] = packed2d(z[f"shared_{n}_packed"], srows[n])
        d[f"{pre}.shared_experts.{PROJ[n]}.scales"] = torch.from_numpy(z[f"shared_{n}_scales"])
    g = torch.Generator().manual_seed(5)
    ln_w = 1.0 + 0.1 * torch.randn(H, generator=g)
    ln_b = 0.05 * torch.randn(H, generator=g)
    if with_norm3:
        d["layers.3.post_attention_layernorm.weight"] = ln_w
        d["layers.3.post_attention_layernorm.bias"] = ln_b
    save_file(d, str(path))
    return z, E, H, I, Is, T, ln_w, ln_b


def test_config_deduced_from_tensor_shapes(tmp_path):
    # deduce_config (src/loader.rs:77-184): router shape -> E, H; a per-expert
    # gate_proj's packed shape -> I, H = 4 x bytes per row; top_k 6; layers =
    # last index + 1
    f = tmp_path / "model.safetensors"
    z, E, H, I, Is, T, _, _ = write_model(f)
    cfg = loader.moe_config_from_tensors(str(f))
    assert (cfg.num_experts, cfg.top_k, cfg.hidden_dim, cfg.intermediate_dim) == (E, 6, H, I)
    assert loader.layer_count(str(f)) == 4


def test_config_json_defaults(tmp_path):
    # parse_config_json (src/loader.rs:186-201): alternative key names and
    # the reference's defaults for the fields the file leaves out
    p = tmp_path / "config.json"
    p.write_text('{"hidden_size": 7168, "num_hidden_layers": 61, "num_local_experts": 256, '
                 '"num_experts_per_tok": 8, "intermediate_size": 2048}')
    cfg, nl = loader.moe_config_from_json(str(p))
    assert (cfg.num_experts, cfg.top_k, cfg.hidden_dim, cfg.intermediate_dim, nl) == (256, 8, 7168, 2048, 61)
    p.write_text("{}")
    cfg, nl = loader.moe_config_from_json(str(p))
    assert (cfg.num_experts, cfg.top_k, cfg.hidden_dim, cfg.intermediate_dim, nl) == (64, 6, 2048, 1408, 27)


def test_post_attention_norm_read_or_identity(tmp_path):
    f = tmp_path / "model.safetensors"
    z, E, H, I, Is, T, ln_w, ln_b = write_model(f)
    w, b = loader.read_norm(str(f), 3, H)
    assert torch.equal(w, ln_w.float()) and torch.equal(b, ln_b.float())
    w0, b0 = loader.read_norm(str(f), 0, H)          # not in the file: ones, zeros
    assert torch.equal(w0, torch.ones(H)) and torch.equal(b0, torch.zeros(H))
    with pytest.raises(ValueError):
        loader.read_norm(str(f), 3, 2 * H)


@pytest.mark.gpu
def test_loaded_block_chain_matches_blocks_and_oracle(tmp_path):
    # the file's two layers (flattened layer 0, per-expert layer 3) chained
    # from one call, against the blocks one by one and the oracle
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from oracle import oracle as qo
    f = tmp_path / "model.safetensors"
    z, E, H, I, Is, T, ln_w, ln_b = write_model(f)
    cfg = MoEConfig(E, 2, H, I)
    x = torch.from_numpy(z["x"]).cuda()
    blocks = [loader.load_block(str(f), l, cfg) for l in (0, 3)]
    ref = x
    for blk in blocks:
        ref = blk.forward_block(ref)
    chain = loader.load_block_chain(str(f), cfg, layers=[0, 3])
    out = chain.forward(x)
    assert torch.equal(out, ref)
    # the oracle: layer 0 = x + FFN(LN0(x)) with the identity norm; layer 3 the block
    np_sh = [(z[f"shared_{n}_packed"].reshape(-1), z[f"shared_{n}_scales"]) for n in ("gate", "up", "down")]
    np_exp = [[(z[f"e{e}_{n}_packed"].reshape(-1), z[f"e{e}_{n}_scales"]) for n in ("gate", "up", "down")]
              for e in range(E)]
    xs = z["x"].astype(np.float32)
    h0 = xs + qo.shared_forward(np_sh, qo.layernorm(xs, np.ones(H, np.float32), np.zeros(H, np.float32)), H, Is)
    h3 = qo.block_forward(qo.MoEConfig(E, 2, H, I, Is), z["gate_w"], np_exp, h0, ln_w.numpy(), ln_b.numpy(),
                          shared=np_sh)
    h3 = h3[0] if isinstance(h3, tuple) else h3
    err = float(np.max(np.abs(out.cpu().numpy() - h3)) / np.max(np.abs(h3)))
    assert err <= 1e-4
    for blk in blocks:
        blk.close()
    chain.close()
