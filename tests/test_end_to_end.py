"""OracleSparseMLP / OracleMLPPatcher: host logic on CPU, selection parity on the GPU."""
from __future__ import annotations

import inspect

import numpy as np
import pytest
import torch
from torch import nn

from conftest import load_npz
from qcc_b200.end_to_end import OracleMLPPatcher, OracleSparseMLP, compute_down_column_norms_chunked, find_gated_mlps


class TinyFFN(nn.Module):
    def __init__(self, h=4, n=8):
        super().__init__()
        self.gate_proj = nn.Linear(h, n, bias=False)
        self.up_proj = nn.Linear(h, n, bias=False)
        self.down_proj = nn.Linear(n, h, bias=False)
        self.act_fn = nn.SiLU()

    def forward(self, x):
        return self.down_proj(self.act_fn(self.gate_proj(x)) * self.up_proj(x))


class Layer(nn.Module):
    def __init__(self, h=4, n=8):
        super().__init__()
        self.mlp = TinyFFN(h, n)
        self.attn_norm = nn.LayerNorm(h)


class Model(nn.Module):
    def __init__(self, layers=3, h=4, n=8):
        super().__init__()
        self.backbone = nn.Module()
        self.backbone.layers = nn.ModuleList([Layer(h, n) for _ in range(layers)])
        self.heads = nn.ModuleList([nn.Linear(h, h)])

    def forward(self, x):
        for layer in self.backbone.layers:
            x = x + layer.mlp(x)
        return x


def test_full_retention_is_identity_and_lazy():
    torch.manual_seed(1)
    mlp = TinyFFN()
    wrapper = OracleSparseMLP(mlp, 0, 1.0)
    x = torch.randn(3, 4)
    wrapper.set_mode(False)
    dense = wrapper(x)
    wrapper.set_mode(True)
    torch.testing.assert_close(wrapper(x), dense)
    assert wrapper.norm_computation_count == 0 and wrapper.down_column_norms is None


def test_forward_is_x_only():
    assert list(inspect.signature(OracleSparseMLP.forward).parameters) == ["self", "x"]


@torch.no_grad()
def test_chunked_norms_match_fp32_for_dtypes_and_chunks():
    torch.manual_seed(8)
    base = torch.randn(97, 521)
    for dtype in (torch.float16, torch.bfloat16, torch.float32):
        weight = base.to(dtype)
        reference = torch.linalg.vector_norm(weight.float(), dim=0)
        for columns in (17, 64, 256, 521, 600):
            torch.testing.assert_close(compute_down_column_norms_chunked(weight, columns), reference,
                                       rtol=1e-6, atol=1e-6)


def test_sparse_mode_on_cpu_fails_loudly():
    wrapper = OracleSparseMLP(TinyFFN(), 0, 0.5)
    wrapper.set_mode(True)
    with pytest.raises(RuntimeError, match="CUDA"):
        wrapper(torch.randn(2, 4))


def test_retention_validation():
    wrapper = OracleSparseMLP(TinyFFN(), 0)
    with pytest.raises(ValueError, match="retention"):
        wrapper.set_mode(True, 0.0)
    with pytest.raises(ValueError):
        OracleSparseMLP(TinyFFN(), 0, norm_chunk_columns=0)


def test_patcher_discovers_wraps_and_restores():
    model = Model()
    assert find_gated_mlps(model) == [f"backbone.layers.{i}.mlp" for i in range(3)]
    originals = [layer.mlp for layer in model.backbone.layers]
    patcher = OracleMLPPatcher(model)
    assert all(isinstance(layer.mlp, OracleSparseMLP) for layer in model.backbone.layers)
    x = torch.randn(2, 4)
    patcher.dense()
    dense = model(x)
    patcher.apply_schedule([1.0, 1.0, 1.0])
    torch.testing.assert_close(model(x), dense)
    with pytest.raises(ValueError, match="schedule"):
        patcher.apply_schedule([1.0])
    patcher.restore()
    assert [layer.mlp for layer in model.backbone.layers] == originals
    assert all(len(m.down_proj._forward_pre_hooks) == 0 for m in originals)


@pytest.mark.gpu
def test_oracle_mlp_matches_reference_golden():
    data = load_npz("oracle_mlp.npz")
    h, n = data["gate"].shape[1], data["gate"].shape[0]
    mlp = TinyFFN(h, n).cuda()
    with torch.no_grad():
        mlp.gate_proj.weight.copy_(torch.from_numpy(data["gate"]))
        mlp.up_proj.weight.copy_(torch.from_numpy(data["up"]))
        mlp.down_proj.weight.copy_(torch.from_numpy(data["down"]))
    wrapper = OracleSparseMLP(mlp, 0, 0.25, norm_chunk_columns=7)
    x = torch.from_numpy(data["x"]).cuda()
    wrapper.set_mode(True, 0.25)
    with torch.no_grad():
        sparse = wrapper(x)
    assert np.array_equal(wrapper.last_selected_indices.cpu().numpy(), data["selected"])
    np.testing.assert_allclose(wrapper.down_column_norms.cpu().numpy(), data["norms"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(sparse.cpu().numpy(), data["sparse"], rtol=1e-5, atol=1e-6)
    wrapper.set_mode(False)
    np.testing.assert_allclose(wrapper(x).detach().cpu().numpy(), data["dense"], rtol=1e-5, atol=1e-6)


@pytest.mark.gpu
def test_accelerate_interception_and_telemetry_on_gpu():
    mlp = TinyFFN(16, 48).cuda()
    down = mlp.down_proj
    old_forward = down.forward
    down._old_forward = old_forward
    down._hf_hook = object()
    events = []

    def accelerate_forward(*args, **kwargs):
        events.append("materialised")
        return down._old_forward(*args, **kwargs)

    down.forward = accelerate_forward
    seen = []
    wrapper = OracleSparseMLP(mlp, 0, 0.75, telemetry=lambda layer, m: seen.append((layer, sorted(m))))
    wrapper.set_mode(True)
    with torch.no_grad():
        wrapper(torch.randn(2, 16, device="cuda"))
    assert events == ["materialised"] and wrapper.norm_computation_count == 1
    assert seen and seen[0][0] == 0 and "relative_l2" in seen[0][1]
    assert wrapper.last_selected_indices.shape == (2, 36)
    wrapper.close()
    assert down._old_forward is old_forward


@pytest.mark.gpu
def test_patched_model_runs_sparse_on_gpu():
    torch.manual_seed(3)
    model = Model(layers=2, h=16, n=64).cuda()
    patcher = OracleMLPPatcher(model)
    patcher.apply_schedule([0.25, 0.5])
    with torch.no_grad():
        y = model(torch.randn(4, 16, device="cuda"))
    assert y.shape == (4, 16)
    assert patcher.norm_computation_count == 2
    assert patcher.wrappers[0].last_selected_indices.shape == (4, 16)
    patcher.restore()


@pytest.mark.gpu
def test_oracle_mlp_full_layer_size_bf16():
    """hidden 5120, N 17408, bf16, 6 rows: selection bit-exact on the reference's score formula."""
    from oracle.select import topk_ids

    torch.manual_seed(5)
    mlp = TinyFFN(5120, 17408).to(device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        for lin in (mlp.gate_proj, mlp.up_proj, mlp.down_proj):
            lin.weight.normal_(0.0, 0.02)
    wrapper = OracleSparseMLP(mlp, 3, 0.25)
    wrapper.set_mode(True)
    x = torch.randn(2, 3, 5120, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        y = wrapper(x)
        a = mlp.act_fn(mlp.gate_proj(x)) * mlp.up_proj(x)
    norms = wrapper.down_column_norms
    np.testing.assert_allclose(norms.cpu().numpy(),
                               torch.linalg.vector_norm(mlp.down_proj.weight.detach().float(), dim=0).cpu().numpy(),
                               rtol=2e-6)
    scores = (a.abs().float() * norms).reshape(-1, 17408).cpu().numpy()
    k = 4352
    want = topk_ids(scores, k)
    got = wrapper.last_selected_indices.reshape(-1, k).cpu().numpy()
    assert np.array_equal(got, want)
    sparse = torch.zeros_like(a).reshape(-1, 17408)
    idx = torch.from_numpy(want).long().cuda()
    sparse.scatter_(1, idx, a.reshape(-1, 17408).gather(1, idx))
    with torch.no_grad():
        expected = torch.nn.functional.linear(sparse.reshape(a.shape), mlp.down_proj.weight)
    assert torch.equal(y, expected)
    wrapper.close()
