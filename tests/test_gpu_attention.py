"""GPU parity of decode attention (split-K flash decoding) and RoPE through the C ABI.

The reference computes attention in FP64; the GPU path is FP32 and must stay within the
north_star tolerance, |gpu - ref| <= 1e-5 * |ref| + 1e-6, against the oracle on the same inputs.
The reference's own operator fixtures use 2e-6 + 2e-6 * |ref|; both are asserted where they apply.
"""
import numpy as np
import pytest

from golden_util import attention_boundary_inputs, bits_equal, golden, north_star_close, operator_close, seeded_normal

pytestmark = pytest.mark.gpu

TOL_REL, TOL_ABS = 1e-5, 1e-6


@pytest.fixture(scope="module")
def sat():
    from satori_b200 import build
    build.build()
    import satori_b200
    return satori_b200


@pytest.fixture(scope="module")
def ctx(sat):
    return sat.default_context(0)


def _close(gpu, ref, what):
    ok = north_star_close(gpu, ref, TOL_REL, TOL_ABS)
    bad = np.flatnonzero(~ok)
    assert ok.all(), (what, bad[:5], gpu[bad[:5]], ref[bad[:5]])


def test_transformer_v2_gqa_fixture(sat, ctx):
    """QwenOperatorTests.GroupedQueryAttentionMatchesReference (QwenOperatorTests.cs:28-43)."""
    a = golden()["transformer_v2"]["gqa"]
    out = sat.TransformerOps.grouped_attention(a["query"], a["keys"], a["values"], a["query_heads"], a["kv_heads"],
                                               a["head_dim"], a["tokens"], ctx=ctx)
    assert operator_close(out, a["output"])


def test_transformer_v1_mha_fixture(sat, ctx):
    """TransformerOpsTests.cs:24: 2 heads x 48, 7 tokens."""
    g = golden()["transformer_v1"]
    out = sat.TransformerOps.attention(g["query"], g["keys"], g["values"], 48, 7, ctx=ctx)
    assert operator_close(out, g["attention"])


def test_attention_boundary_fixture(sat, ctx):
    """attention-boundaries-v1.json: 6 heads x 48, tokens 1, 2, 32, 64, 128."""
    q, k, v = attention_boundary_inputs()
    for case in golden()["attention_boundaries_v1"]["cases"]:
        t = case["count"]
        out = sat.TransformerOps.attention(q, k[:t].ravel(), v[:t].ravel(), 48, t, ctx=ctx)
        assert operator_close(out, case["expected"]), t


def test_extreme_values_take_the_fp64_path(sat, ctx):
    """TransformerOpsTests.cs:33-36: FLT_MAX queries/keys overflow FP32 scores; the result is still [3, 4]."""
    fmax = np.finfo(np.float32).max
    q = np.array([fmax, fmax], np.float32)
    k = np.array([fmax, fmax, -fmax, -fmax], np.float32)
    out = sat.TransformerOps.attention(q, k, np.array([3, 4, 100, 200], np.float32), 2, 2, ctx=ctx)
    np.testing.assert_array_equal(out, np.array([3, 4], np.float32))


def test_overflowing_head_in_the_streaming_kernel_takes_the_fp64_path(sat, ctx, oracle_lib):
    """28/4 x 128 (the streaming kernel and its fused split merge): one head's FP32 scores overflow, so
    that head is recomputed in FP64 inside the merging CTA; every head stays within tolerance."""
    qh, kvh, hd, tokens = 28, 4, 128, 300
    q = seeded_normal(41, qh * hd)
    k = seeded_normal(42, tokens * kvh * hd)
    v = seeded_normal(43, tokens * kvh * hd)
    q[3 * hd:4 * hd] = 1e19                                # head 3 reads KV head 0
    k[(5 * kvh + 0) * hd:(5 * kvh + 1) * hd] = 1e19        # token 5 of KV head 0: score ~1e39 overflows
    gpu = sat.TransformerOps.grouped_attention(q, k, v, qh, kvh, hd, tokens, ctx=ctx)
    ref = oracle_lib.grouped_attention(q, k, v, qh, kvh, hd, tokens, threads=8)
    _close(gpu, ref, "overflow")
    np.testing.assert_allclose(gpu[3 * hd:4 * hd], v[(5 * kvh) * hd:(5 * kvh + 1) * hd], rtol=1e-6)


def test_equal_heads_equals_mha_bitwise(sat, ctx):
    """QwenOperatorTests.cs:45-60."""
    rng = np.random.default_rng(11)
    q, k, v = (rng.random(n).astype(np.float32) for n in (8, 24, 24))
    a = sat.TransformerOps.grouped_attention(q, k, v, 2, 2, 4, 3, ctx=ctx)
    b = sat.TransformerOps.attention(q, k, v, 4, 3, ctx=ctx)
    assert bits_equal(a, b)


def test_invalid_dimensions_rejected(sat, ctx):
    """QwenOperatorTests.InvalidGroupedAttentionDimensionsAreRejected (:96-104)."""
    q, k = np.zeros(32, np.float32), np.zeros(48, np.float32)
    with pytest.raises(sat.ArgumentError):
        sat.TransformerOps.grouped_attention(q, k, k, 4, 3, 8, 3, ctx=ctx)
    with pytest.raises(sat.ArgumentError):
        sat.TransformerOps.rope_half(np.zeros(8, np.float32), 8, 0, 10000, 5, ctx=ctx)


@pytest.mark.parametrize("key", ["rope_full", "rope_partial"])
def test_rope_half_fixtures(sat, ctx, key):
    """QwenOperatorTests.HalfSplitRopeMatchesReference (:62-76)."""
    r = golden()["transformer_v2"][key]
    v = np.array(r["input"], np.float32)
    sat.TransformerOps.rope_half(v, r["head_dim"], r["position"], r["base"], r["rotary"], ctx=ctx)
    assert operator_close(v, r["output"])


@pytest.mark.parametrize("tokens", [1, 2, 31, 33, 129, 512, 1000, 4096])
@pytest.mark.parametrize("shape", [(28, 4), (12, 2), (8, 8), (6, 1)])
def test_gqa_random_within_north_star_tolerance(sat, ctx, oracle_lib, tokens, shape):
    """BASELINE config 3 geometry (28/4 x 128) plus 1.5B (12/2), MHA and MQA, N(0,1) q/k/v."""
    qh, kvh = shape
    hd = 128
    q = seeded_normal(tokens, qh * hd)
    k = seeded_normal(tokens + 1, tokens * kvh * hd)
    v = seeded_normal(tokens + 2, tokens * kvh * hd)
    gpu = sat.TransformerOps.grouped_attention(q, k, v, qh, kvh, hd, tokens, ctx=ctx)
    ref = oracle_lib.grouped_attention(q, k, v, qh, kvh, hd, tokens, threads=8)
    _close(gpu, ref, (shape, tokens))


def test_gqa_32k_context_within_tolerance(sat, ctx, oracle_lib):
    """BASELINE config 3 at its largest context (T = 32768), with RoPE'd q as in decode."""
    qh, kvh, hd, T = 28, 4, 128, 32768
    q = seeded_normal(1, qh * hd)
    k = seeded_normal(2, T * kvh * hd)
    v = seeded_normal(3, T * kvh * hd)
    q = oracle_lib.rope_half(q, hd, T - 1, 1e6, hd)
    gpu = sat.TransformerOps.grouped_attention(q, k, v, qh, kvh, hd, T, ctx=ctx)
    ref = oracle_lib.grouped_attention(q, k, v, qh, kvh, hd, T, threads=8)
    _close(gpu, ref, "32k")


def test_attention_cache_step_matches_reference_sequence(sat, ctx, oracle_lib):
    """DenseForward.cs:135-143: RopeHalf q/k at the position, append k/v, attend over pos+1 tokens."""
    qh, kvh, hd, steps = 12, 2, 128, 40
    cache = sat.AttentionCache(layers=2, context=64, q_heads=qh, kv_heads=kvh, head_dim=hd, rope_base=1e6, ctx=ctx)
    keys = np.zeros((steps, kvh * hd), np.float32)
    values = np.zeros((steps, kvh * hd), np.float32)
    for pos in range(steps):
        q = seeded_normal(10 * pos + 1, qh * hd)
        k = seeded_normal(10 * pos + 2, kvh * hd)
        v = seeded_normal(10 * pos + 3, kvh * hd)
        gpu = cache.append(1, pos, q, k, v)
        qr = oracle_lib.rope_half(q, hd, pos, 1e6, hd)
        keys[pos] = oracle_lib.rope_half(k, hd, pos, 1e6, hd)
        values[pos] = v
        ref = oracle_lib.grouped_attention(qr, keys[:pos + 1].ravel(), values[:pos + 1].ravel(), qh, kvh, hd, pos + 1)
        _close(gpu, ref, pos)
    with pytest.raises(sat.ContextFullError):
        cache.append(0, 64, q, k, v)
