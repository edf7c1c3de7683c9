"""The FreeToken bridge's runtime factory and ``triton_indexed_ffn``, through the reference's names.

FreeToken itself is not installed; as in the reference's own bridge tests
(tests/test_freetoken_qcc.py:11-31, a fake MLP and a fake runtime) the bridge
is faked: ``FakeBridge`` keeps what ``FreeTokenQCCBridge`` does with its
factory (integration/freetoken_qcc/bridge.py:179-205, 212-257) -- build the
runtime once, lazily, under a lock, route decode rows [1, hidden] to
``runtime.run(x)`` and everything else to the original forward.  Here the
runtime is the real engine (``QCCBridgeRuntime``) on small synthetic
weights and a predictor checkpoint in the reference's format.
"""
from __future__ import annotations

import threading
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import ffn as offn
from oracle import predictor as opred
from oracle.select import topk_ids

H, N, LATENT = 512, 1024, 32


class FakeBridge:
    def __init__(self, config, runtime_factory):
        self.config = config
        self.runtime_factory = runtime_factory
        self._runtime = None
        self._lock = threading.Lock()
        self.counters = {"sparse_decode_calls": 0, "dense_fallback_calls": 0}

    @property
    def runtime(self):
        if self._runtime is None:
            with self._lock:
                if self._runtime is None:
                    self._runtime = self.runtime_factory(self.config)
        return self._runtime

    def forward(self, original, instance, x):
        if x.ndim != 2 or tuple(x.shape) != (1, H):
            self.counters["dense_fallback_calls"] += 1
            return original(instance, x)
        y, _ = self.runtime.run(x)
        self.counters["sparse_decode_calls"] += 1
        return y


def _checkpoint(tmp_path, seed=3):
    g = torch.Generator().manual_seed(seed)
    model = {
        "encoder.weight": torch.randn(LATENT, H, generator=g) * 0.05,
        "residual_fc1.weight": torch.randn(LATENT, LATENT, generator=g) * 0.2,
        "residual_fc1.bias": torch.randn(LATENT, generator=g) * 0.1,
        "residual_fc2.weight": torch.randn(LATENT, LATENT, generator=g) * 0.2,
        "residual_fc2.bias": torch.randn(LATENT, generator=g) * 0.1,
        "layer_norm.weight": 1 + 0.1 * torch.randn(LATENT, generator=g),
        "layer_norm.bias": 0.1 * torch.randn(LATENT, generator=g),
        "neurons.weight": torch.randn(N, LATENT, generator=g) * 0.3,
        "neurons.bias": torch.randn(N, generator=g) * 0.1,
    }
    ckpt = {"config": {"kind": "residual_factorized", "input_dim": H, "output_dim": N, "latent_dim": LATENT},
            "model": model, "mean": torch.randn(H, generator=g) * 0.1, "std": 0.5 + torch.rand(H, generator=g)}
    path = tmp_path / "best.pt"
    torch.save(ckpt, path)
    return path, ckpt


def _weights(tmp_path, dtype=torch.float16, seed=4):
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(seed)
    gate = (torch.randn(N, H, generator=g) * 0.02).to(dtype)
    up = (torch.randn(N, H, generator=g) * 0.02).to(dtype)
    down = (torch.randn(H, N, generator=g) * 0.02).to(dtype)
    path = tmp_path / "layer.safetensors"
    save_file({"gate_proj.weight": gate, "up_proj.weight": up, "down_proj.weight": down}, str(path),
              metadata={"source": "synthetic"})
    return path, (gate, up, down)


def _config(ckpt, weights, **kw):
    base = dict(mode="replace", layer=0, selector_checkpoint=ckpt, runtime_weights=weights, variant="warp8",
                retention=0.5)
    base.update(kw)
    return SimpleNamespace(**base)


def test_runtime_refuses_cpu_input_and_unknown_variant(tmp_path):
    from qcc_b200.integration.freetoken import QCCBridgeRuntime, runtime_factory

    assert runtime_factory is QCCBridgeRuntime
    rt = QCCBridgeRuntime(_config(tmp_path / "a.pt", tmp_path / "w.safetensors"))
    with pytest.raises(RuntimeError, match="requires a CUDA input tensor"):
        rt.run(torch.zeros(1, H))
    assert not rt.initialized


def test_triton_name_checks_before_any_gpu_work():
    from qcc_b200.runtime import triton_indexed_ffn
    from qcc_b200.runtime.triton_sparse_ffn import TRITON_AVAILABLE

    assert TRITON_AVAILABLE is False
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        triton_indexed_ffn(torch.zeros(1, 8), torch.zeros(2, dtype=torch.long), torch.zeros(4, 8), torch.zeros(4, 8),
                           torch.zeros(8, 4))


@pytest.mark.gpu
@pytest.mark.parametrize("packed_artefact", [False, True])
def test_bridge_runtime_factory_end_to_end(tmp_path, packed_artefact):
    from qcc_b200.integration.freetoken import make_runtime_factory
    from qcc_b200.runtime import artefact

    ckpt_path, ckpt = _checkpoint(tmp_path)
    w_path, (gate, up, down) = _weights(tmp_path)
    if packed_artefact:
        artefact.pack_safetensors_layer(w_path, tmp_path / "packed")
        w_path = tmp_path / "packed"
    constructions = []

    def factory(config):
        constructions.append(config)
        return make_runtime_factory(expected_shape=(H, N))(config)

    bridge = FakeBridge(_config(ckpt_path, w_path), factory)
    mlp = SimpleNamespace(calls=0)

    def original(instance, x):
        instance.calls += 1
        return x + 1

    g = torch.Generator().manual_seed(9)
    xs = [torch.randn(1, H, generator=g).to(torch.bfloat16).cuda() for _ in range(3)]
    outs = [bridge.forward(original, mlp, x) for x in xs]
    prefill = torch.zeros(4, H, device="cuda")
    assert torch.equal(bridge.forward(original, mlp, prefill), prefill + 1)
    torch.cuda.synchronize()
    assert len(constructions) == 1 and mlp.calls == 1
    assert bridge.counters == {"sparse_decode_calls": 3, "dense_fallback_calls": 1}
    rt = bridge.runtime
    rt.check()
    assert rt.memory["ffn_weight_bytes"] == N * 3 * H * 2
    # Selection: the oracle predictor on the checkpoint, normalisation folded, fp16 weights.
    w, b = opred.fold_normalisation(ckpt["model"]["encoder.weight"].numpy(), ckpt["mean"].numpy(),
                                    ckpt["std"].numpy())
    p = {"enc_w": w, "enc_b": b}
    for name, key in (("fc1_w", "residual_fc1.weight"), ("fc1_b", "residual_fc1.bias"),
                      ("fc2_w", "residual_fc2.weight"), ("fc2_b", "residual_fc2.bias"),
                      ("ln_w", "layer_norm.weight"), ("ln_b", "layer_norm.bias"), ("out_w", "neurons.weight"),
                      ("out_b", "neurons.bias")):
        p[name] = ckpt["model"][key].numpy()
    p16 = {k: torch.as_tensor(np.asarray(v, dtype=np.float32)).half().double().numpy() for k, v in p.items()}
    k = N // 2
    for x, y in zip(xs, outs):
        assert y.dtype == x.dtype and y.shape == (1, H)
        y2, ids = rt.run(x)
        assert torch.equal(y2, y)
        scores = rt.selector.run(x.half())[0]
        assert np.array_equal(ids.cpu().numpy(), topk_ids(scores.cpu().numpy(), k)[0])
        ref_scores = opred.predictor_scores(x.half().double().cpu().numpy(), p16, "residual", 1e-5)
        assert np.abs(scores.double().cpu().numpy() - ref_scores).max() <= 1e-3 * max(1.0, np.abs(ref_scores).max())
        want = offn.sparse_ffn_f64(x.half().cpu(), ids.long().cpu(), gate, up, down)
        assert offn.rel_l2(y.double().cpu().numpy(), want) <= 1e-2


@pytest.mark.gpu
def test_bridge_runtime_rejects_shape_and_device_mismatch(tmp_path):
    from qcc_b200.integration.freetoken import QCCBridgeRuntime, make_runtime_factory

    ckpt_path, _ = _checkpoint(tmp_path)
    w_path, _ = _weights(tmp_path)
    with pytest.raises(ValueError, match="expected"):
        QCCBridgeRuntime(_config(ckpt_path, w_path)).run(torch.zeros(1, H, device="cuda"))
    with pytest.raises(ValueError, match="Unknown CUDA indexed variant"):
        QCCBridgeRuntime(_config(ckpt_path, w_path, variant="nope"), expected_shape=(H, N)).run(
            torch.zeros(1, H, device="cuda"))
    rt = make_runtime_factory(expected_shape=(H, N))(_config(ckpt_path, w_path))
    rt.run(torch.zeros(1, H, device="cuda"))
    if torch.cuda.device_count() > 1:
        with pytest.raises(RuntimeError, match="initialized on"):
            rt.run(torch.zeros(1, H, device="cuda:1"))


@pytest.mark.gpu
@pytest.mark.parametrize("transposed_down", [False, True])
def test_triton_indexed_ffn_matches_oracle(transposed_down):
    from qcc_b200.runtime import triton_indexed_ffn

    g = torch.Generator().manual_seed(5)
    gate = (torch.randn(300, 64, generator=g) * 0.05).bfloat16()
    up = (torch.randn(300, 64, generator=g) * 0.05).bfloat16()
    down = (torch.randn(64, 300, generator=g) * 0.05).bfloat16()
    x = torch.randn(1, 64, generator=g).bfloat16()
    ids = torch.randperm(300, generator=g)[:70]
    d = down.t().contiguous() if transposed_down else down
    y = triton_indexed_ffn(x.cuda(), ids.cuda(), gate.cuda(), up.cuda(), d.cuda(), transposed_down=transposed_down)
    want = offn.dynamic_sparse_ffn(x, ids, gate, up, down)
    assert y.shape == (1, 64) and y.dtype == torch.bfloat16
    assert offn.rel_l2(y.double().cpu().numpy(), want.double().numpy()) <= 1e-2
    with pytest.raises(ValueError, match="batch=1"):
        triton_indexed_ffn(torch.cat([x, x]).cuda(), ids.cuda(), gate.cuda(), up.cuda(), d.cuda(), transposed_down)
    with pytest.raises(ValueError, match="down weight shape must be"):
        triton_indexed_ffn(x.cuda(), ids.cuda(), gate.cuda(), up.cuda(), d.t().contiguous().cuda(), transposed_down)
