"""GPU parity of the HiF8 token embedding (gather-decode of the requested
rows) and of projections loaded from an exported-format checkpoint.

* embedding: bit-exact against the CPU oracle and the golden fixture made by
  the reference's own lookup (scheme.py:120-131), NaN patterns aside; the
  vectorised (hidden % 16 == 0) and scalar kernels, through the PyTorch
  operator and through the C ABI; out-of-range ids.
* checkpoint: fused qkv / gate_up / in_proj_qkvz linears and single
  projections loaded onto the GPU, static quant + linear at decode and
  prefill row counts within max-rel 1e-2 of the FP64 oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests._helpers import bf16_bits, max_rel
from tests.test_checkpoint_cpu import make_checkpoint
from tests.test_oracle_golden import assert_bf16_equal_nan_any

pytestmark = pytest.mark.gpu
GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"
DEV = "cuda:0"


def _embed(w: np.ndarray, ws: np.ndarray, ids: np.ndarray, *, via_cabi: bool = False, validate: bool = False):
    from hif8_b200 import cabi, checkpoint

    weight = torch.from_numpy(np.ascontiguousarray(w)).to(DEV)
    scale = torch.from_numpy(np.ascontiguousarray(ws, dtype=np.float32).reshape(-1)).to(DEV)
    tid = torch.from_numpy(np.ascontiguousarray(ids, dtype=np.int64)).to(DEV)
    if via_cabi:
        out = torch.empty(*tid.shape, weight.shape[1], dtype=torch.bfloat16, device=DEV)
        bad = torch.zeros(1, dtype=torch.int32, device=DEV)
        cabi.embedding_gather(weight, scale, tid, out, bad)
        torch.cuda.synchronize()
        return bf16_bits(out), int(bad.item())
    out = checkpoint.Hif8Embedding(weight, scale)(tid, validate=validate)
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16 and out.shape == (*ids.shape, w.shape[1])
    return bf16_bits(out), 0


@pytest.mark.parametrize("via_cabi", [False, True])
@pytest.mark.parametrize("case", ["ka", "v", "s"])
def test_embedding_matches_reference_fixture(case, via_cabi):
    g = np.load(GOLDEN / "embedding.npz")
    w, ws, ids = g[f"{case}_w"], g[f"{case}_ws"], g[f"{case}_ids"]
    out, bad = _embed(w, ws, ids, via_cabi=via_cabi)
    assert bad == 0
    assert_bf16_equal_nan_any(out, g[f"{case}_out"])
    # and exactly the oracle's bits (canonical NaN included)
    np.testing.assert_array_equal(out, oracle.embedding(w, ws, ids))


@pytest.mark.parametrize("hidden", [4096, 2560, 48, 7])
def test_embedding_random_rows_bit_exact(hidden):
    rng = np.random.default_rng(hidden)
    vocab = 1000
    w = rng.integers(0, 256, size=(vocab, hidden), dtype=np.uint8)
    ws = (np.abs(rng.standard_normal(vocab)) * 1e-3 + 1e-7).astype(np.float32)
    for ids in (rng.integers(0, vocab, size=(4,)), rng.integers(0, vocab, size=(3, 17)), np.array([vocab - 1, 0, 0])):
        out, _ = _embed(w, ws, ids)
        np.testing.assert_array_equal(out, oracle.embedding(w, ws, ids))
        out_c, _ = _embed(w, ws, ids, via_cabi=True)
        np.testing.assert_array_equal(out_c, out)


def test_embedding_out_of_range_ids():
    rng = np.random.default_rng(5)
    w = rng.integers(0, 256, size=(64, 32), dtype=np.uint8)
    ws = np.full(64, 0.5, np.float32)
    ids = np.array([3, 64, -1, 63])
    out, bad = _embed(w, ws, ids, via_cabi=True)
    assert bad == 2
    np.testing.assert_array_equal(out, oracle.embedding(w, ws, ids))
    assert not out[1].any() and not out[2].any()
    with pytest.raises(IndexError, match="outside the vocabulary"):
        _embed(w, ws, ids, validate=True)
    out, _ = _embed(w, ws, np.zeros((0,), np.int64))
    assert out.shape == (0, 32)


@pytest.mark.parametrize("m", [1, 4, 8, 40])
def test_checkpoint_linears_on_gpu_match_oracle(tmp_path, m):
    from hif8_b200 import checkpoint

    make_checkpoint(tmp_path, seed=m)
    ckpt = checkpoint.Hif8Checkpoint(tmp_path)
    layers = [ckpt.fused_linear("model.layers.0", "self_attn", "qkv_proj", DEV),
              ckpt.fused_linear("model.layers.0", "mlp", "gate_up_proj", DEV),
              ckpt.fused_linear("model.layers.1", "linear_attn", "in_proj_qkvz", DEV),
              ckpt.linear("model.layers.0.self_attn.o_proj", DEV),
              ckpt.linear("model.layers.0.mlp.down_proj", DEV)]
    g = torch.Generator().manual_seed(m)
    for layer in layers:
        x = (torch.randn(m, layer.in_features, generator=g) * 20).to(torch.bfloat16)
        y = layer(x.to(DEV)).float().cpu().numpy()
        s = layer.input_scale.cpu().numpy()
        a, a_s = oracle.static_quant(bf16_bits(x), s)
        ref = oracle.linear(a, layer.weight.cpu().numpy(), a_s, layer.weight_scale.cpu().numpy())
        assert y.shape == (m, layer.out_features)
        assert max_rel(y, ref) <= 1e-2, f"{layer.out_features}x{layer.in_features} M={m}"


def test_checkpoint_embedding_on_gpu(tmp_path):
    from hif8_b200 import checkpoint

    tensors = make_checkpoint(tmp_path)
    emb = checkpoint.Hif8Checkpoint(tmp_path).embedding(DEV)
    ids = torch.tensor([[1, 31, 0], [7, 7, 2]], dtype=torch.int64)
    out = emb(ids.to(DEV))
    expected = oracle.embedding(tensors["model.embed_tokens.weight"].numpy(),
                                tensors["model.embed_tokens.weight_scale"].numpy(), ids.numpy())
    np.testing.assert_array_equal(bf16_bits(out), expected)
