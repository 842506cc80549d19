"""Pin the CPU oracle: the reference's own known-answer tests restated, plus agreement with an
independent numpy restatement of the full forward step.  CPU only."""
import math

import numpy as np
import pytest

from oracle import oracle as O


# ---------------------------------------------------------------- reference KATs
def test_rope_freqs_values_kat():
    """RotationTests.computeRopeFreqsValues (engine/ml/src/test/java/org/almostrealism/ml/RotationTests.java:511-532):
    theta 1e4, headDim 8, seqLen 4: freqCis[pos,f] = (cos, sin)(pos * theta^(-2f/headDim)) within 1e-6."""
    theta, head_dim, seq_len = 10000.0, 8, 4
    for prec in ("f64", "f32"):
        fc = O.rope_freqs(theta, head_dim, seq_len, prec)
        for pos in range(seq_len):
            for f in range(head_dim // 2):
                ang = pos * math.pow(theta, -2.0 * f / head_dim)
                assert abs(fc[pos, f, 0] - math.cos(ang)) < 1e-6
                assert abs(fc[pos, f, 1] - math.sin(ang)) < 1e-6


def test_rope_freqs_qwen_theta():
    fc = O.rope_freqs(1e6, 128, 1024)
    pos = np.arange(1024)[:, None]
    inv = 1e6 ** (-2.0 * np.arange(64) / 128)
    np.testing.assert_allclose(fc[..., 0], np.cos(pos * inv), atol=1e-9)
    np.testing.assert_allclose(fc[..., 1], np.sin(pos * inv), atol=1e-9)


def test_gqa_expand_kat():
    """GQAExpandTest.testGQAExpand (engine/ml/src/test/java/org/almostrealism/ml/qwen3/GQAExpandTest.java:27-101):
    input[kv*headSize + h] = kv*1000 + h; every query head reproduces its kv head."""
    heads, kv_heads, hs = 14, 2, 64
    x = np.array([(i // hs) * 1000 + (i % hs) for i in range(kv_heads * hs)], np.float64)
    out = O.gqa_expand(x, kv_heads, heads, hs)
    for h in range(heads):
        base = (h // (heads // kv_heads)) * 1000
        for i in range(hs):
            assert abs(out[h * hs + i] - (base + i)) <= 0.001


def test_causal_mask_kat():
    """CausalMaskIsolationTest (engine/ml/src/test/java/org/almostrealism/ml/CausalMaskIsolationTest.java:26-60):
    heads 4, seqLen 8; at position 0 column 0 is unchanged and column 1 gets -10000 (tol 1e-6, FP64)."""
    rng = np.random.default_rng(3)
    x = rng.random((4, 8))
    for pos in range(8):
        y = O.causal_mask(x, pos)
        for h in range(4):
            for t in range(8):
                want = x[h, t] + (-10000.0 if t > pos else 0.0)
                assert abs(y[h, t] - want) < 1e-6


def test_attention_keys_kat():
    """AttentionTests.attentionKeys (engine/ml/src/test/java/org/almostrealism/ml/AttentionTests.java:51-96):
    seqLength 128, heads 12, headSize 64 against the explicit loop."""
    rng = np.random.default_rng(5)
    S, H, d = 128, 12, 64
    q, K = rng.random((H, d)), rng.random((S, H, d))
    att = O.attention_keys(q, K)
    for h in range(H):
        for t in range(S):
            score = sum(q[h, i] * K[t, h, i] for i in range(d)) / math.sqrt(d)
            assert abs(score - att[h, t]) < 1e-12


def test_attention_values_kat():
    """AttentionTests.attentionValues (AttentionTests.java:103-152): seqLength 1024, heads 12, headSize 64."""
    rng = np.random.default_rng(6)
    S, H, d = 1024, 12, 64
    a, V = rng.random((H, S)), rng.random((S, H, d))
    out = O.attention_values(a, V)
    want = np.einsum("hs,shi->hi", a, V)
    np.testing.assert_allclose(out, want, rtol=1e-12)
    h, i = 7, 33
    assert abs(sum(a[h, t] * V[t, h, i] for t in range(S)) - out[h, i]) < 1e-9


def test_softmax_log_stable():
    """softmax with subtractMax (ActivationFeatures.java:136-142): exp(x - m - log sum exp(x - m))."""
    rng = np.random.default_rng(7)
    x = rng.normal(size=(3, 50)) * 30
    y = O.softmax(x)
    e = np.exp(x - x.max(1, keepdims=True))
    np.testing.assert_allclose(y, e / e.sum(1, keepdims=True), rtol=1e-12)
    # -10000 masked entries get exactly zero weight
    x[:, 10:] -= 10000.0
    assert np.all(O.softmax(x)[:, 10:] == 0.0)


def test_rmsnorm_formula():
    rng = np.random.default_rng(8)
    x, w = rng.normal(size=64), rng.normal(size=64)
    y = O.rmsnorm(x, w, 1e-6)
    np.testing.assert_allclose(y, w * x / np.sqrt((x * x).sum() / 64 + 1e-6), rtol=1e-13)


def test_argmax_first_max():
    """indexOfMax keeps the first maximum (strict greaterThan, AggregationFeatures.java:111-121)."""
    v = np.array([1, 5, 3, 5, 5, -1], np.float32)
    assert O.argmax(v) == 1
    assert O.argmax(np.zeros(10, np.float32)) == 0


def test_synth_generator_moments():
    scale = 0.02 / math.sqrt(4.0 * (65536.0 ** 2 - 1) / 12.0)
    vals = np.array([O.synth_value(0, 16 + 2, i, scale) for i in range(20000)])
    assert abs(vals.mean()) < 0.02 * 0.05
    assert abs(vals.std() - 0.02) < 0.02 * 0.05
    assert O.synth_value(0, 18, 123, scale) == O.synth_value(0, 18, 123, scale)
    assert O.synth_value(0, 18, 123, scale) != O.synth_value(1, 18, 123, scale)


# ---------------------------------------------------------------- independent numpy restatement
def numpy_forward_model(sd, cfg, tokens):
    """Straight numpy restatement of the reference step (fp64), full seqLen cache with the -10000
    mask, GQA-expanded cache, whole-vector QK-norm; returns logits per position."""
    D, H, Hkv, d, S = cfg["dim"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"], cfg["seq_len"]
    g = H // Hkv
    f = {k: np.asarray(v, np.float64) for k, v in sd.items()}
    inv = np.exp(np.arange(d // 2) * (-2.0 * math.log(cfg["rope_theta"]) / d))
    kc = np.zeros((cfg["layers"], S, H, d))
    vc = np.zeros((cfg["layers"], S, H, d))

    def rms(x, w, eps):
        return w * x / np.sqrt((x * x).sum() / x.size + eps)

    def rope(x, pos):
        x = x.reshape(-1, d).copy()
        c, s = np.cos(pos * inv), np.sin(pos * inv)
        a, b = x[:, : d // 2].copy(), x[:, d // 2:].copy()
        x[:, : d // 2] = a * c - b * s
        x[:, d // 2:] = b * c + a * s
        return x

    out = []
    for pos, t in enumerate(tokens):
        x = f["model.embed_tokens.weight"][t].copy()
        for l in range(cfg["layers"]):
            p = f"model.layers.{l}."
            a = rms(x, f[p + "input_layernorm.weight"], 1e-6)
            q = f[p + "self_attn.q_proj.weight"] @ a
            k = f[p + "self_attn.k_proj.weight"] @ a
            v = f[p + "self_attn.v_proj.weight"] @ a
            q = rms(q, f[p + "self_attn.q_norm.weight"].ravel(), 1e-6)
            k = rms(k, f[p + "self_attn.k_norm.weight"].ravel(), 1e-6)
            q, k = rope(q, pos), rope(k, pos)
            kc[l, pos] = np.repeat(k, g, axis=0)
            vc[l, pos] = np.repeat(v.reshape(-1, d), g, axis=0)
            s = np.einsum("hd,thd->ht", q, kc[l]) / math.sqrt(d)
            s = s + np.where(np.arange(S) > pos, -10000.0, 0.0)[None]
            s = np.exp(s - s.max(1, keepdims=True))
            s /= s.sum(1, keepdims=True)
            o = np.einsum("ht,thd->hd", s, vc[l]).ravel()
            x = x + f[p + "self_attn.o_proj.weight"] @ o
            b = rms(x, f[p + "post_attention_layernorm.weight"], 1e-6)
            g1 = f[p + "mlp.gate_proj.weight"] @ b
            u = f[p + "mlp.up_proj.weight"] @ b
            x = x + f[p + "mlp.down_proj.weight"] @ (u * g1 / (1 + np.exp(-g1)))
        wcls = f.get("lm_head.weight", f["model.embed_tokens.weight"])
        out.append(wcls @ rms(x, f["model.norm.weight"], 1e-6))
    return np.array(out)


TINY = dict(dim=64, hidden_dim=96, layers=2, heads=4, kv_heads=2, head_dim=16, vocab=97, seq_len=12,
            shared_weights=0, qk_norm=1, rope_theta=1e6, eps=1e-6)


def tiny_state_dict(cfg, seed=0, std=0.2, norm_noise=True):
    rng = np.random.default_rng(seed)
    D, Q, KV, F, V = cfg["dim"], cfg["heads"] * cfg["head_dim"], cfg["kv_heads"] * cfg["head_dim"], cfg["hidden_dim"], cfg["vocab"]
    n = lambda *s: (rng.standard_normal(s) * std).astype(np.float32)  # noqa: E731
    ones = lambda *s: (1 + (rng.standard_normal(s) * 0.1 if norm_noise else 0)).astype(np.float32)  # noqa: E731
    sd = {"model.embed_tokens.weight": n(V, D), "model.norm.weight": ones(D), "lm_head.weight": n(V, D)}
    for l in range(cfg["layers"]):
        p = f"model.layers.{l}."
        sd.update({p + "input_layernorm.weight": ones(D), p + "post_attention_layernorm.weight": ones(D),
                   p + "self_attn.q_proj.weight": n(Q, D), p + "self_attn.k_proj.weight": n(KV, D),
                   p + "self_attn.v_proj.weight": n(KV, D), p + "self_attn.o_proj.weight": n(D, Q),
                   p + "self_attn.q_norm.weight": ones(cfg["heads"], cfg["head_dim"]),
                   p + "self_attn.k_norm.weight": ones(cfg["kv_heads"], cfg["head_dim"]),
                   p + "mlp.gate_proj.weight": n(F, D), p + "mlp.up_proj.weight": n(F, D),
                   p + "mlp.down_proj.weight": n(D, F)})
    return sd


def test_oracle_matches_numpy_restatement():
    sd = tiny_state_dict(TINY)
    toks = [3, 17, 50, 2, 96, 0, 41, 41, 7, 8, 9, 10]
    want = numpy_forward_model(sd, TINY, toks)
    m = O.OracleModel(TINY, "f64")
    m.load_state_dict(sd)
    got = np.array([m.forward_token(t, p) for p, t in enumerate(toks)])
    np.testing.assert_allclose(got, want.astype(np.float32), rtol=1e-5, atol=1e-6)


def test_oracle_f32_close_to_f64():
    sd = tiny_state_dict(TINY)
    toks = [1, 2, 3, 4, 5, 6]
    a, b = O.OracleModel(TINY, "f64"), O.OracleModel(TINY, "f32")
    a.load_state_dict(sd)
    b.load_state_dict(sd)
    for p, t in enumerate(toks):
        la, lb = a.forward_token(t, p), b.forward_token(t, p)
        assert np.linalg.norm(la - lb) / np.linalg.norm(la) < 1e-5


def test_oracle_generate_matches_stepwise():
    """AutoregressiveModel.next(): prompt fed one per step, then argmax of the previous logits."""
    sd = tiny_state_dict(TINY)
    m = O.OracleModel(TINY, "f64")
    m.load_state_dict(sd)
    toks, _ = m.generate([5, 6, 7], 10)
    m.reset()
    cur, out = None, []
    for s in range(10):
        t = [5, 6, 7][s] if s < 3 else O.argmax(cur)
        out.append(t)
        cur = m.forward_token(t, s)
    assert list(toks) == out


def test_oracle_reset_clears_cache():
    sd = tiny_state_dict(TINY)
    m = O.OracleModel(TINY, "f64")
    m.load_state_dict(sd)
    a = [m.forward_token(t, p) for p, t in enumerate([4, 5, 6])]
    m.reset()
    b = [m.forward_token(t, p) for p, t in enumerate([4, 5, 6])]
    np.testing.assert_array_equal(np.array(a), np.array(b))


def test_oracle_rejects_bad_inputs():
    m = O.OracleModel(TINY, "f64")
    with pytest.raises(ValueError):
        m.forward_token(TINY["vocab"], 0)
    with pytest.raises(ValueError):
        m.forward_token(0, TINY["seq_len"])
    with pytest.raises(ValueError):
        m.set("model.layers.0.self_attn.q_proj.weight", np.zeros(3, np.float32))


def test_golden_fixture_regression():
    """The committed fixture (tests/golden/make_golden.py) still matches the oracle."""
    import os
    path = os.path.join(os.path.dirname(__file__), "golden", "tiny_f64.npz")
    g = np.load(path)
    sd = tiny_state_dict(TINY)
    m = O.OracleModel(TINY, "f64")
    m.load_state_dict(sd)
    got = np.array([m.forward_token(t, p) for p, t in enumerate(g["tokens"])])
    np.testing.assert_allclose(got, g["logits"], rtol=1e-6, atol=1e-7)


# ---------------------------------------------------------------- sampling restatements
def test_java_random_known_answers():
    """java.util.Random known answers: new Random(0).nextDouble(), new Random(42).nextDouble() (twice) and
    new Random(42).nextInt()."""
    r = O.JavaRandom(0)
    assert r.next_double() == 0.730967787376657
    r = O.JavaRandom(42)
    assert r.next_double() == 0.7275636800328681
    assert r.next_double() == 0.6832234717598454
    assert O.JavaRandom(42).next(32) == -1170105035


def test_sample_token_matches_direct_loops():
    """sampleToken restated with numpy against a literal loop transcription of its steps."""
    rng = np.random.default_rng(11)
    for trial in range(20):
        V = 50
        logits = rng.normal(size=V) * 3
        T, top_p, r = [0.7, 1.3][trial % 2], [0.3, 0.9, 1.0][trial % 3], rng.random()
        probs = [x / T for x in logits]
        m = max(probs)
        probs = [math.exp(x - m) for x in probs]
        s = sum(probs)
        probs = [x / s for x in probs]
        if top_p < 1.0:
            idx = sorted(range(V), key=lambda i: -probs[i])
            cum = 0.0
            top_sum = 0.0
            cutoff = V
            for i in range(V):
                cum += probs[idx[i]]
                top_sum += probs[idx[i]]
                if cum >= top_p:
                    cutoff = i + 1
                    break
            for i in range(cutoff, V):
                probs[idx[i]] = 0.0
            probs = [x / top_sum for x in probs]
        want, c = V - 1, 0.0
        for i in range(V):
            c += probs[i]
            if r < c:
                want = i
                break
        assert O.sample_token(logits, V, T, top_p, r) == want


def test_sample_greedy_and_ties():
    v = np.array([0.5, 2.0, 2.0, -1.0])
    assert O.sample_token(v, 4, 0.0, 1.0, 0.3) == 1
    assert O.sample_qwen3(v, 4, 0.0, 0.3) == 1
    # equal probabilities keep index order inside the nucleus: the two tied maxima at top_p 0.4
    v = np.array([1.0, 3.0, 3.0, 0.0])
    assert O.sample_token(v, 4, 1.0, 0.4, 0.999) == 1
