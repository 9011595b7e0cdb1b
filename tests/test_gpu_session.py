"""GPU decode session vs the oracle's DenseSession restatement, through the C ABI.

Projections are bit-exact to the reference; RMSNorm, RoPE and SwiGLU follow its FP64 formulas;
attention is FP32 within 1e-5 relative + 1e-6 absolute.  Logits therefore agree to a small
tolerance, and greedy tokens must be identical (north_star: "greedy decode tokens must be
identical on the small configs").
"""
import numpy as np
import pytest

import os

from model_util import device_synthetic_tensors, synthetic_tensors

pytestmark = pytest.mark.gpu

# Stated tolerance on logits after a full forward step.  Projections are bit-exact and RmsNorm, RoPE and
# SwiGLU follow the reference's FP64 formulas; attention runs in FP32 (within 1e-5 rel + 1e-6 abs of the
# reference's FP64), and that difference, carried through up to 28 layers, reaches ~1.5e-5 absolute on
# the 7B shape's near-zero logits.  The reference's own whole-model checks allow 1e-3 + 1e-3 |x|
# (QwenForwardTests.cs:113) and 5e-3 + 5e-3 |x| (:60); this bound is 20-100x tighter.
LOGIT_REL, LOGIT_ABS = 1e-4, 5e-5


@pytest.fixture(scope="module")
def sat():
    from satori_b200 import build
    build.build()
    import satori_b200
    return satori_b200


@pytest.fixture(scope="module")
def ctx(sat):
    return sat.default_context(0)


def _run_pair(sat, ctx, spec, prompt, n_gen, context=64, seed=7, tensors=None):
    from oracle.oracle import OracleSession
    tensors = tensors if tensors is not None else synthetic_tensors(spec, seed)
    gpu = sat.CudaDenseSession(spec, tensors, context, ctx=ctx)
    ref = OracleSession(spec, tensors, context)
    threads = max(8, os.cpu_count() or 1)
    tok = None
    greedy = []
    for i in range(len(prompt) + n_gen):
        t = int(prompt[i]) if i < len(prompt) else tok
        lg, ag = gpu.append(t)
        lr, ar = ref.append(t, threads=threads)
        err = np.abs(lg.astype(np.float64) - lr)
        assert np.all(err <= LOGIT_REL * np.abs(lr) + LOGIT_ABS), (i, float(err.max()))
        assert ag == ar, (i, ag, ar)
        greedy.append(ag)
        tok = ar
    return gpu, ref, greedy


@pytest.mark.parametrize("fmt", [0, 1])
def test_tiny_model_logits_and_greedy_tokens(sat, ctx, oracle_lib, fmt):
    spec = sat.tiny(proj_format=fmt)
    gpu, ref, _ = _run_pair(sat, ctx, spec, prompt=[1, 5, 9, 200, 3], n_gen=20)
    assert gpu.position == ref.position == 25
    np.testing.assert_allclose(gpu.stage(0), ref.stage(0), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(gpu.stage(1), ref.stage(1), rtol=1e-4, atol=1e-5)


def test_gqa_without_bias_and_tied_embeddings(sat, ctx, oracle_lib):
    spec = sat.tiny(layers=3, q_heads=8, kv_heads=1, head_dim=32, hidden=256, has_bias=False)
    spec.tied_embeddings = True
    tensors = synthetic_tensors(spec, 3)
    tensors["output.weight"] = tensors["token_embd.weight"]   # the oracle reads the tied matrix by this name
    _run_pair(sat, ctx, spec, prompt=[4], n_gen=11, context=32, tensors=tensors)


def test_generate_matches_stepwise_greedy(sat, ctx, oracle_lib):
    """Device-side greedy loop equals step-by-step appends; reset restores the fresh state bitwise."""
    spec = sat.tiny()
    tensors = synthetic_tensors(spec, 11)
    s = sat.CudaDenseSession(spec, tensors, 64, ctx=ctx)
    first_logits, _ = s.append(3)
    s.reset()
    assert s.position == 0
    again, _ = s.append(3)
    assert np.array_equal(first_logits.view(np.uint32), again.view(np.uint32))
    s.reset()
    gen = s.generate(3, 16)
    s.reset()
    steps, t = [], 3
    for _ in range(16):
        _, t = s.append(t)
        steps.append(t)
    assert list(gen) == steps


def test_session_errors(sat, ctx, oracle_lib):
    """DenseSession.Append's checks (DenseSession.cs:113-117) and the Q4_0 embedding rejection."""
    spec = sat.tiny()
    tensors = synthetic_tensors(spec, 5)
    s = sat.CudaDenseSession(spec, tensors, 4, ctx=ctx)
    with pytest.raises(sat.ArgumentError):
        s.append(spec.vocab)
    with pytest.raises(sat.ArgumentError):
        s.append(-1)
    for t in range(4):
        s.append(t)
    with pytest.raises(sat.ContextFullError):
        s.append(0)
    s.dispose()
    with pytest.raises(sat.DisposedError):
        s.append(0)
    bad = sat.tiny()
    bad.embd_format = 1
    t2 = dict(tensors)
    t2["token_embd.weight"] = oracle_lib.q_quantize(np.zeros(bad.vocab * bad.hidden, np.float32), bad.vocab,
                                                    bad.hidden, 1)
    with pytest.raises(sat.NotSupportedError):
        sat.CudaDenseSession(bad, t2, 4, ctx=ctx)


def test_qwen2_1_5b_config_128_prompt_256_greedy_tokens_identical(sat, ctx, oracle_lib):
    """BASELINE config 4 as stated (28 layers, 1536 hidden, 12/2 heads, FFN 8960, vocab 151936, all
    Q8_0; a 128-token seeded prompt, then 256 greedy tokens): every step's logits are within tolerance
    of the oracle's and every greedy token is identical (DenseSession.cs:111-131)."""
    spec = sat.qwen2_1_5b()
    tensors = device_synthetic_tensors(ctx, spec, seed=21)
    prompt = list(np.random.default_rng(4).integers(0, spec.vocab, 128))
    gpu, ref, greedy = _run_pair(sat, ctx, spec, prompt=prompt, n_gen=256, context=400, tensors=tensors)
    assert gpu.position == ref.position == 384
    gpu.dispose()
    ref.close()


def test_qwen2_7b_shape_session_matches_oracle(sat, ctx, oracle_lib):
    """BASELINE config 5 shape on one GPU (28 layers, 3584 hidden, 28/4 heads, FFN 18944, vocab
    152064; Q4_0 projections, Q8_0 embedding and lm_head): 4 prompt tokens + 8 greedy tokens, logits
    within tolerance and greedy tokens identical to the oracle's at every step."""
    spec = sat.qwen2_7b()
    tensors = device_synthetic_tensors(ctx, spec, seed=31)
    prompt = list(np.random.default_rng(8).integers(0, spec.vocab, 4))
    gpu, ref, _ = _run_pair(sat, ctx, spec, prompt=prompt, n_gen=8, context=16, tensors=tensors)
    gpu.dispose()
    ref.close()


def test_rewind_replays_identically(sat, ctx, oracle_lib):
    """satori_session_rewind keeps the cache below the position: decoding again from there gives the
    same tokens bitwise, and a rewind past the committed position is refused."""
    spec = sat.tiny()
    s = sat.CudaDenseSession(spec, synthetic_tensors(spec, 13), 64, ctx=ctx)
    s.prefill([5, 9, 17, 2])
    first = s.generate(7, 12)
    s.rewind(4)
    again = s.generate(7, 12)
    assert list(first) == list(again) and s.position == 16
    with pytest.raises(sat.ArgumentError):
        s.rewind(17)
    info = s.info()
    assert info["kernels_per_step"] > 0 and info["weight_bytes"] > 0
    assert info["kv_bytes_per_position"] == spec.layers * 2 * spec.kv_width * 4


@pytest.mark.parametrize("fmt", [0, 1])
def test_fused_projections_match_separate_launches_bitwise(sat, ctx, oracle_lib, fmt, monkeypatch):
    """q/k/v stacked into one launch and gate/up interleaved with the SwiGLU epilogue give the same
    bits as the separate launches (each row keeps its own FP32 chain; SwiGLU is the same function)."""
    spec = sat.tiny(proj_format=fmt)           # hidden 256: the gate/up pair takes the fused epilogue
    tensors = synthetic_tensors(spec, 9)
    fused = sat.CudaDenseSession(spec, tensors, 32, ctx=ctx)
    monkeypatch.setenv("SATORI_FUSE", "0")
    apart = sat.CudaDenseSession(spec, tensors, 32, ctx=ctx)
    t = 5
    for _ in range(12):
        a, ta = fused.append(t)
        b, tb = apart.append(t)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)) and ta == tb
        t = ta


def test_session_from_gguf_equals_session_from_tensors(sat, ctx, oracle_lib, tmp_path):
    """A qwen2 GGUF file loaded natively (satori_session_create_from_gguf: catalogue, model shape, uploads
    from the mapping) steps bit for bit like a session built from the same tensors."""
    import gguf_util
    spec = sat.tiny(proj_format=1)
    tensors = synthetic_tensors(spec, 17)
    path = tmp_path / "tiny.gguf"
    path.write_bytes(gguf_util.model_gguf(spec, tensors))
    a = sat.session_from_gguf(str(path), 32, ctx=ctx)
    b = sat.CudaDenseSession(spec, tensors, 32, ctx=ctx)
    t = 9
    for _ in range(10):
        la, ta = a.append(t)
        lb, tb = b.append(t)
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32)) and ta == tb
        t = ta
    a.dispose()
    b.dispose()
