"""GPU tests of the tensor-core prefill path (SATORI_ORDER_TENSOR).

DenseSession.Forward prefills a chunk through DenseForward.LayerBatch, whose projections are
QuantizedMatVec.ExecuteBatch over the chunk's positions (QuantizedMatVec.cs:221-365).  On the GPU that
product is a GEMM on tcgen05.  It is not the reference's FP32 operation order, so these tests bound it
instead of comparing bits:

* against an FP64 decode-and-dot, every output stays within the worst-case bound of ANY FP32
  summation order of the row (gamma_n * sum|w x|, n = cols + cols/32 + 2 -- the bound the reference's
  own ExecuteBatch result satisfies) plus 2^-24 * sum|w x| for the activation split (x is carried as
  three bf16 parts, exact to 2^-27 |x|; the dropped cross products are below 2^-25 of |w x| each);
* against the oracle's ExecuteBatch restatement, the difference stays within twice that bound.
"""
import numpy as np
import pytest

from golden_util import gamma_bound, seeded_normal

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sat():
    from satori_b200 import build
    build.build()
    import satori_b200
    return satori_b200


@pytest.fixture(scope="module")
def ctx(sat):
    return sat.default_context(0)


def _decode(payload: np.ndarray, rows: int, cols: int, fmt: int) -> np.ndarray:
    """GgufQuantizedMatrix row decode in FP64 (d * q, exact)."""
    bb = 34 if fmt == 0 else 18
    bpr = cols // 32
    p = payload.reshape(rows, bpr, bb)
    d = p[:, :, 0:2].copy().view(np.float16).astype(np.float64).reshape(rows, bpr)
    if fmt == 0:
        q = p[:, :, 2:].view(np.int8).astype(np.float64)
    else:
        qb = p[:, :, 2:].astype(np.int32)
        q = np.concatenate([(qb & 15) - 8, (qb >> 4) - 8], axis=2).astype(np.float64)
    return (d[:, :, None] * q).reshape(rows, cols)


def _random_payload(rng, rows: int, cols: int, fmt: int) -> np.ndarray:
    bb = 34 if fmt == 0 else 18
    payload = rng.integers(0, 256, size=rows * (cols // 32) * bb, dtype=np.uint8)
    scales = (rng.standard_normal(rows * (cols // 32)) * 0.05).astype(np.float16).view(np.uint16)
    p2 = payload.reshape(-1, bb)
    p2[:, 0] = scales & 0xFF
    p2[:, 1] = scales >> 8
    return payload


def _check_bound(y, payload, rows, cols, fmt, x, positions, what):
    w = _decode(payload, rows, cols, fmt)
    xs = x.astype(np.float64).reshape(positions, cols)
    exact = xs @ w.T                       # [positions][rows]
    mag = np.abs(xs) @ np.abs(w).T
    bound = gamma_bound(cols, mag) + 2.0 ** -24 * mag
    err = np.abs(y.reshape(positions, rows).astype(np.float64) - exact)
    worst = float(np.max(err / np.maximum(bound, 1e-300)))
    assert np.all(err <= bound), (what, worst, np.argwhere(err > bound)[:4])
    return bound


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("rows,cols,positions", [(1, 64, 1), (7, 128, 3), (128, 64, 16), (300, 4096, 7),
                                                  (129, 1536, 17), (1003, 896, 33), (3584, 3584, 128),
                                                  (18944, 1024, 9), (256, 18944, 130)])
def test_tensor_order_within_fp32_bound(sat, ctx, fmt, rows, cols, positions):
    """Random payloads (every code value, random scales): single tiles, partial row tiles, split-K
    (few row tiles) and unsplit (many row tiles) launches, and more than one 128-position chunk."""
    rng = np.random.default_rng(rows * 31 + cols + positions + fmt)
    payload = _random_payload(rng, rows, cols, fmt)
    x = rng.standard_normal(positions * cols).astype(np.float32)
    m = sat.CudaMatrixFactory(ctx).create(payload, sat.QuantizedMatrixShape(rows, cols, fmt))
    y = m.execute_tensor(x, positions)
    assert y.shape == (positions * rows,) and np.all(np.isfinite(y))
    _check_bound(y, payload, rows, cols, fmt, x, positions, "fp64")
    m.dispose()


@pytest.mark.parametrize("fmt", [0, 1])
def test_tensor_order_close_to_execute_batch(sat, ctx, oracle_lib, fmt):
    """Quantized N(0, 0.02^2) weights (the model-like case) against the oracle's ExecuteBatch order."""
    rows, cols, positions = 512, 3584, 24
    w = seeded_normal(40 + fmt, rows * cols, 0.02)
    payload = oracle_lib.q_quantize(w, rows, cols, fmt)
    x = seeded_normal(41 + fmt, positions * cols)
    m = sat.CudaMatrixFactory(ctx).create(payload, sat.QuantizedMatrixShape(rows, cols, fmt))
    y = m.execute_tensor(x, positions)
    bound = _check_bound(y, payload, rows, cols, fmt, x, positions, "fp64")
    ref = oracle_lib.q_matvec(payload, rows, cols, fmt, x, order="batch", positions=positions, threads=8)
    diff = np.abs(y.astype(np.float64) - ref.astype(np.float64)).reshape(positions, rows)
    assert np.all(diff <= 2 * bound)
    # The tensor order agrees with the decode order to FP32 level, far inside the bound.
    assert np.max(diff / np.maximum(bound, 1e-300)) < 0.25


def test_tensor_order_rejections(sat, ctx):
    rng = np.random.default_rng(5)
    tern = sat.Ternary2Matrix.quantize(rng.standard_normal(64 * 64).astype(np.float32), 64, 64, 64, ctx=ctx)
    with pytest.raises(sat.NotSupportedError):
        tern.device.execute_tensor(np.ones(64, np.float32), 1)
    payload = _random_payload(rng, 4, 96, 0)       # 96 columns: not a multiple of 64
    m = sat.CudaMatrixFactory(ctx).create(payload, sat.QuantizedMatrixShape(4, 96, 0))
    with pytest.raises(sat.NotSupportedError):
        m.execute_tensor(np.ones(96 * 2, np.float32), 2)
    out = np.full(8, 7.0, np.float32)
    with pytest.raises(sat.NotSupportedError):
        m.execute_tensor(np.ones(96 * 2, np.float32), 2, out)
    assert np.all(out == 7.0)


# ---------------------------------------------------------------- session prefill (satori_session_forward_tensor)
# The prefill's projections differ from ExecuteBatch's FP32 order by a few roundings of sum|w x| (bounded
# above), so every cache row it writes differs from the per-token path's at that level, and the difference
# is carried through every layer and every later position's attention.  Measured on the 1.5B shape (28
# layers, 200 prefilled positions): 7.1e-5 absolute on the logits, against 1.7e-5 for the per-token path.
# The stated bound is 1e-4 relative + 2e-4 absolute, five times tighter than the reference's own
# whole-model check (1e-3 + 1e-3 |x|, QwenForwardTests.cs:113); greedy tokens must be identical.
LOGIT_REL, LOGIT_ABS = 1e-4, 2e-4


def _close(a, b):
    err = np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))
    return bool(np.all(err <= LOGIT_REL * np.abs(np.asarray(b, np.float64)) + LOGIT_ABS)), float(err.max())


def _prefill_vs_oracle(sat, ctx, spec, tensors, prompt, n_gen, context):
    import os
    from oracle.oracle import OracleSession
    threads = max(8, os.cpu_count() or 1)
    gpu = sat.CudaDenseSession(spec, tensors, context, ctx=ctx)
    ref = OracleSession(spec, tensors, context)
    lg = gpu.forward(prompt, tensor_cores=True)
    for t in prompt:
        lr, ar = ref.append(int(t), threads=threads)
    ok, worst = _close(lg, lr)
    assert ok, ("prefill logits", worst)
    print(f"prefill {spec.name}: worst logit error {worst:.3g}")
    tok = int(np.argmax(lr))
    assert int(np.argmax(lg)) == tok
    assert gpu.position == ref.position == len(prompt)
    for i in range(n_gen):
        lg, ag = gpu.append(tok)
        lr, ar = ref.append(tok, threads=threads)
        ok, worst = _close(lg, lr)
        assert ok and ag == ar, (i, worst, ag, ar)
        tok = ar
    gpu.dispose()
    ref.close()


@pytest.mark.parametrize("fmt", [0, 1])
def test_tiny_prefill_matches_oracle(sat, ctx, oracle_lib, fmt):
    """Two full 128-position chunks and a ragged one (300 prompt tokens), then 16 greedy tokens."""
    from model_util import synthetic_tensors
    spec = sat.tiny(proj_format=fmt)
    prompt = np.random.default_rng(50 + fmt).integers(0, spec.vocab, 300)
    _prefill_vs_oracle(sat, ctx, spec, synthetic_tensors(spec, 51), prompt, 16, 340)


def test_prefill_gqa_without_bias_and_tied_embeddings(sat, ctx, oracle_lib):
    """8 query heads on one KV head (head_dim 32: the general attention kernel), no q/k/v bias."""
    from model_util import synthetic_tensors
    spec = sat.tiny(layers=3, q_heads=8, kv_heads=1, head_dim=32, hidden=256, has_bias=False)
    spec.tied_embeddings = True
    tensors = synthetic_tensors(spec, 3)
    tensors["output.weight"] = tensors["token_embd.weight"]
    prompt = np.random.default_rng(52).integers(0, spec.vocab, 37)
    _prefill_vs_oracle(sat, ctx, spec, tensors, prompt, 8, 64)


def test_prefill_after_decoded_prefix_and_separate_projections(sat, ctx, oracle_lib, monkeypatch):
    """A prefill that starts mid-context (positions already decoded) with q/k/v and gate/up kept apart."""
    import os
    from model_util import synthetic_tensors
    from oracle.oracle import OracleSession
    monkeypatch.setenv("SATORI_FUSE", "0")
    spec = sat.tiny(proj_format=1)
    tensors = synthetic_tensors(spec, 53)
    gpu = sat.CudaDenseSession(spec, tensors, 256, ctx=ctx)
    ref = OracleSession(spec, tensors, 256)
    threads = max(8, os.cpu_count() or 1)
    head = [7, 1, 99, 4, 250]
    for t in head:
        gpu.append(t)
        ref.append(t, threads=threads)
    rest = np.random.default_rng(54).integers(0, spec.vocab, 140)
    lg = gpu.forward(rest, tensor_cores=True)
    for t in rest:
        lr, _ = ref.append(int(t), threads=threads)
    ok, worst = _close(lg, lr)
    assert ok and int(np.argmax(lg)) == int(np.argmax(lr)), worst
    assert gpu.position == ref.position == 145
    gpu.dispose()
    ref.close()


def test_prefill_errors_commit_nothing(sat, ctx, oracle_lib):
    from model_util import synthetic_tensors
    spec = sat.tiny()
    s = sat.CudaDenseSession(spec, synthetic_tensors(spec, 55), 40, ctx=ctx)
    s.forward([1, 2, 3], tensor_cores=True)
    with pytest.raises(sat.ArgumentError):
        s.forward([1, spec.vocab, 3], tensor_cores=True)
    with pytest.raises(sat.ContextFullError):
        s.forward(list(range(38)), tensor_cores=True)
    assert s.position == 3
    one = s.forward([9], tensor_cores=True)          # one token: the decode step alone
    assert s.position == 4 and np.all(np.isfinite(one))


def test_qwen2_1_5b_prefill_matches_oracle(sat, ctx, oracle_lib):
    """BASELINE config 4 weights (all Q8_0, 12/2 heads x 128): a 200-token prompt in two chunks, then
    16 greedy tokens, against the oracle's DenseSession step by step."""
    from model_util import device_synthetic_tensors
    spec = sat.qwen2_1_5b()
    tensors = device_synthetic_tensors(ctx, spec, seed=21)
    prompt = np.random.default_rng(56).integers(0, spec.vocab, 200)
    _prefill_vs_oracle(sat, ctx, spec, tensors, prompt, 16, 240)


def test_qwen2_7b_shape_prefill_matches_per_token_path(sat, ctx, oracle_lib):
    """BASELINE config 5 shape (Q4_0 projections, 28/4 heads, the streaming attention kernel): a
    300-token tensor-core prefill against the per-token path (itself bit-exact to the oracle's
    projections), then 8 greedy tokens each, identical."""
    from model_util import device_synthetic_tensors
    spec = sat.qwen2_7b()
    tensors = device_synthetic_tensors(ctx, spec, seed=31)
    prompt = np.random.default_rng(57).integers(0, spec.vocab, 300)
    a = sat.CudaDenseSession(spec, tensors, 320, ctx=ctx)
    b = sat.CudaDenseSession(spec, tensors, 320, ctx=ctx)
    del tensors
    la = a.forward(prompt, tensor_cores=True)
    lb = b.forward(prompt)
    ok, worst = _close(la, lb)
    assert ok and int(np.argmax(la)) == int(np.argmax(lb)), worst
    first = int(np.argmax(lb))
    assert list(a.generate(first, 8)) == list(b.generate(first, 8))
    a.dispose()
    b.dispose()


def test_prefill_with_per_head_norms_matches_per_token_path(sat, ctx, oracle_lib):
    """qwen3-style layers (no q/k/v bias, attn_q_norm / attn_k_norm per head, DenseForward.cs:130-133): the
    chunk's batched head norms against the decode step's (TransformerOps.RmsNormHeads, pinned by the
    reference's qk_norm fixture); logits within the prefill tolerance and greedy tokens identical."""
    from model_util import synthetic_tensors
    spec = sat.tiny(layers=2, q_heads=8, kv_heads=2, head_dim=128, hidden=512, ffn=1024, has_bias=False)
    tensors = synthetic_tensors(spec, 61)
    rng = np.random.default_rng(62)
    for l in range(spec.layers):
        for part in ("q", "k"):
            tensors[f"blk.{l}.attn_{part}_norm.weight"] = (1.0 + 0.1 * rng.standard_normal(spec.head_dim)).astype(
                np.float32)
    prompt = rng.integers(0, spec.vocab, 150)
    a = sat.CudaDenseSession(spec, tensors, 200, ctx=ctx)
    b = sat.CudaDenseSession(spec, tensors, 200, ctx=ctx)
    la = a.forward(prompt, tensor_cores=True)
    lb = b.forward(prompt)
    ok, worst = _close(la, lb)
    assert ok and int(np.argmax(la)) == int(np.argmax(lb)), worst
    first = int(np.argmax(lb))
    assert list(a.generate(first, 10)) == list(b.generate(first, 10))
    a.dispose()
    b.dispose()
