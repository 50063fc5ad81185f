"""The toy MoE decoder -- moe_decoder_* against the CPU
restatement in oracle/decoder_oracle.py.

CPU tests pin the oracle: its RoPE against the reference's own
tensor_ops::apply_rope (src/tensor.cu:191-210, compiled into oracle/_ref),
its attention block against the reference's PhiAttention::forward
(src/layer.cu:110-147, built with plain multi-head attention), its greedy
loop against its own prefill, and its EOS rule (generate_decode,
src/model.cu:2061-2104).  GPU tests run the decoder through the C ABI at a
small shape (2 layers, d 256, vocab 1024, 8 experts top-2) and, for 2 layers,
at config 4's own layer shapes (d 2048, 16 heads, 16 experts of 5632,
vocab 32000), and compare:
  - prefill logits: relative L2 <= 1e-3 in FP32 (3xTF32), <= 3e-2 in BF16
    (every activation rounded to bf16 before each GEMM);
  - greedy ids: equal to the oracle's until the sequences diverge, and a
    divergence only where the oracle's top-2 logit gap is below the
    precision's noise margin (FP32 2e-3, BF16 5e-2); logits at the shared
    prefix within the same bounds as prefill.
"""
import sys

import numpy as np
import pytest

from conftest import ROOT, load_oracle, load_pkg, rel_l2

sys.path.insert(0, str(ROOT / "oracle"))

SMALL = dict(n_layers=2, d=256, vocab=1024, E=8, ff=384)
TOL = {0: 1e-3, 1: 3e-2}          # precision -> rel-L2 bound on logits
MARGIN = {0: 2e-3, 1: 5e-2}       # precision -> top-2 gap a divergence may sit within


def _weights(seed=2, **kw):
    pkg = load_pkg()
    shape = dict(SMALL, **kw)
    return pkg.synthetic_decoder(seed, shape["n_layers"], shape["d"], shape["vocab"], shape["E"],
                                 shape["ff"], norm_jitter=0.1)


def _oracle(w, heads, hd):
    load_oracle()
    import decoder_oracle
    return decoder_oracle.DecoderOracle(w, heads, hd)


# ---------------------------------------------------------------- CPU
def test_oracle_rope_matches_reference_apply_rope():
    orc_mod = load_oracle()
    if not orc_mod.Reference.available(8):
        pytest.skip("reference library not built (reference sources absent)")
    import decoder_oracle
    ref = orc_mod.Reference(8)
    g = np.random.default_rng(5)
    S, H, hd = 48, 3, 64
    q = g.standard_normal((S, H * hd)).astype(np.float32)
    k = g.standard_normal((S, H * hd)).astype(np.float32)
    rq, rk = ref.apply_rope(q, k, H, hd, 10000.0)
    pos = np.arange(S)
    oq = decoder_oracle.apply_rope(q.reshape(S, H, hd).astype(np.float64), pos, hd, 10000.0)
    ok = decoder_oracle.apply_rope(k.reshape(S, H, hd).astype(np.float64), pos, hd, 10000.0)
    # The reference forms each angle in float (pow, then position * inv), the
    # restatement in double: they agree to the float rounding of the angle.
    assert np.max(np.abs(oq.reshape(S, -1) - rq)) < 2e-5
    assert np.max(np.abs(ok.reshape(S, -1) - rk)) < 2e-5


def _write_tensors(path, entries):
    """fp32 tensors in the ModelLoader format (src/model_loader.cu:14-30)."""
    import struct
    metas = [(n.encode(), a.shape, a.nbytes) for n, a in entries]
    hsize = 4 + sum(4 + len(nb) + 4 + 4 * len(sh) + 16 for nb, sh, _ in metas)
    header, off = bytearray(struct.pack("<I", len(entries))), hsize
    for nb, sh, nbytes in metas:
        header += struct.pack("<I", len(nb)) + nb + struct.pack("<I", len(sh))
        header += struct.pack(f"<{len(sh)}I", *sh) + struct.pack("<QQ", off, nbytes)
        off += nbytes
    with open(path, "wb") as f:
        f.write(header)
        for _, a in entries:
            f.write(np.ascontiguousarray(a, np.float32).tobytes())


def test_oracle_attention_matches_reference_phi_attention(tmp_path):
    """The restatement's attention block (projections, rotate-half RoPE,
    causal softmax scaled by 1/sqrt(hd), o projection) against the
    reference's own PhiAttention::forward built with plain multi-head
    attention; zero biases, since config 4 has none."""
    orc_mod = load_oracle()
    if not orc_mod.ReferenceAttention.available():
        pytest.skip("reference attention library not built (reference sources absent)")
    import decoder_oracle
    ref = orc_mod.ReferenceAttention()
    H, hd = ref.heads, 128
    d = H * hd
    g = np.random.default_rng(7)
    w = {n: (0.05 * g.standard_normal((d, d))).astype(np.float32) for n in ("q", "k", "v", "o")}
    entries = []
    for n in ("q", "k", "v", "o"):
        entries.append((f"model.layers.0.self_attn.{n}_proj.weight", w[n]))
        entries.append((f"model.layers.0.self_attn.{n}_proj.bias", np.zeros(d, np.float32)))
    path = tmp_path / "attn.bin"
    _write_tensors(path, entries)
    for S in (1, 17, 40):
        x = g.standard_normal((S, d)).astype(np.float32)
        y_ref = ref.forward(path, 0, x, d)
        y = decoder_oracle.self_attention(x, w["q"], w["k"], w["v"], w["o"], 1, S, H, hd, 10000.0)
        assert rel_l2(y, y_ref) <= 1e-5, (S, rel_l2(y, y_ref))


def test_oracle_greedy_loop_restarts_from_the_prefix():
    import decoder_oracle  # noqa: F401
    w = _weights(n_layers=1, d=128, vocab=256, ff=128)
    o = _oracle(w, 1, 128)
    pkg = load_pkg()
    prompt = pkg.synthetic_prompt(1, 2, 7, w.vocab)
    ids, lg = o.generate(prompt, 3)
    assert np.array_equal(lg[:, 0], o.last_logits(prompt))
    assert np.array_equal(ids[:, 0], np.argmax(lg[:, 0], axis=1))
    ext = np.concatenate([prompt, ids[:, :1]], axis=1)
    assert np.allclose(lg[:, 1], o.last_logits(ext), rtol=0, atol=0)


def test_oracle_stops_a_sequence_at_eos():
    w = _weights(n_layers=1, d=128, vocab=256, ff=128)
    o = _oracle(w, 1, 128)
    pkg = load_pkg()
    prompt = pkg.synthetic_prompt(3, 2, 5, w.vocab)
    ids, _ = o.generate(prompt, 4)
    eos = int(ids[0, 1])
    ids2, lg2 = o.generate(prompt, 4, eos_id=eos)
    stop = int(np.argmax(ids2[0] == eos))
    assert np.all(ids2[0, stop + 1:] == -1) and np.all(lg2[0, stop + 1:] == 0)


# ---------------------------------------------------------------- GPU
def _decoder(w, heads, hd, precision, max_batch=4, max_seq=128):
    pkg = load_pkg()
    return pkg.MoeDecoder(w, n_heads=heads, head_dim=hd, precision=precision,
                          max_batch=max_batch, max_seq=max_seq)


def _check_greedy(ids, lg, ids_ref, lg_ref, precision):
    import decoder_oracle
    B, n = ids.shape
    for b in range(B):
        for t in range(n):
            assert rel_l2(lg[b, t], lg_ref[b, t]) <= TOL[precision], (b, t)
            if ids[b, t] != ids_ref[b, t]:
                gap = decoder_oracle.top2_margin(lg_ref[b, t])
                assert gap <= MARGIN[precision], (b, t, gap)
                break   # the prefixes differ from here on


@pytest.mark.gpu
@pytest.mark.parametrize("precision", [0, 1], ids=["fp32", "bf16"])
@pytest.mark.parametrize("heads,hd", [(2, 128), (4, 64)], ids=["hd128", "hd64"])
def test_decoder_prefill_matches_oracle(precision, heads, hd):
    pkg = load_pkg()
    w = _weights()
    o = _oracle(w, heads, hd)
    prompt = pkg.synthetic_prompt(2, 2, 40, w.vocab)
    ref = o.last_logits(prompt)
    with _decoder(w, heads, hd, precision) as m:
        lg, nxt = m.prefill(prompt)
    assert rel_l2(lg, ref) <= TOL[precision], rel_l2(lg, ref)
    import decoder_oracle
    for b in range(2):
        if nxt[b] != np.argmax(ref[b]):
            assert decoder_oracle.top2_margin(ref[b]) <= MARGIN[precision]


@pytest.mark.gpu
@pytest.mark.parametrize("precision", [0, 1], ids=["fp32", "bf16"])
def test_decoder_generate_matches_oracle(precision):
    pkg = load_pkg()
    w = _weights()
    o = _oracle(w, 2, 128)
    prompt = pkg.synthetic_prompt(4, 3, 33, w.vocab)
    ids_ref, lg_ref = o.generate(prompt, 6)
    with _decoder(w, 2, 128, precision) as m:
        ids, lg = m.generate(prompt, 6)
        pre, dec = m.last_timing()
    assert pre > 0 and dec > 0
    _check_greedy(ids, lg, ids_ref, lg_ref, precision)


@pytest.mark.gpu
@pytest.mark.parametrize("precision", [0, 1], ids=["fp32", "bf16"])
@pytest.mark.parametrize("heads,hd", [(2, 128), (4, 64)], ids=["hd128", "hd64"])
def test_decoder_batch1_generate_matches_oracle(precision, heads, hd):
    """One sequence: every dense projection runs at one row (in BF16 the
    weight-streaming GEMV, one row per pass), the MoE block through the
    small-batch router and the decode kernels."""
    pkg = load_pkg()
    w = _weights()
    o = _oracle(w, heads, hd)
    prompt = pkg.synthetic_prompt(9, 1, 24, w.vocab)
    ids_ref, lg_ref = o.generate(prompt, 6)
    with _decoder(w, heads, hd, precision) as m:
        ids, lg = m.generate(prompt, 6)
    _check_greedy(ids, lg, ids_ref, lg_ref, precision)


@pytest.mark.gpu
@pytest.mark.parametrize("precision", [0, 1], ids=["fp32", "bf16"])
@pytest.mark.parametrize("heads,hd", [(2, 128), (4, 64)], ids=["hd128", "hd64"])
def test_decoder_long_prefill(precision, heads, hd):
    """2 x 200 rows: the projections run the CTA-pair tiles (>= 256 rows) and
    the prefill attention spans two query and two key blocks of 128 (the
    tensor-core kernel in BF16), the causal diagonal crossing a block."""
    pkg = load_pkg()
    w = _weights()
    o = _oracle(w, heads, hd)
    prompt = pkg.synthetic_prompt(5, 2, 200, w.vocab)
    ref = o.last_logits(prompt)
    with _decoder(w, heads, hd, precision, max_seq=256) as m:
        lg, _ = m.prefill(prompt)
        ids, lgg = m.generate(prompt, 3)
    assert rel_l2(lg, ref) <= TOL[precision], rel_l2(lg, ref)
    ids_ref, lg_ref = o.generate(prompt, 3)
    _check_greedy(ids, lgg, ids_ref, lg_ref, precision)


@pytest.mark.gpu
def test_decoder_step_api_matches_generate():
    pkg = load_pkg()
    w = _weights()
    prompt = pkg.synthetic_prompt(6, 2, 20, w.vocab)
    with _decoder(w, 2, 128, 0) as m:
        ids, lg = m.generate(prompt, 4)
        l0, n0 = m.prefill(prompt)
        steps = [(l0, n0)]
        for _ in range(3):
            steps.append(m.decode_step(steps[-1][1]))
    for t, (lt, nt) in enumerate(steps):
        # Decode-sized projections split K with atomic adds: equal up to
        # summation order.
        assert rel_l2(lt, lg[:, t]) <= 1e-5
        assert np.array_equal(nt, ids[:, t])


@pytest.mark.gpu
def test_decoder_eos_stops_a_sequence():
    pkg = load_pkg()
    w = _weights()
    prompt = pkg.synthetic_prompt(7, 2, 16, w.vocab)
    with _decoder(w, 2, 128, 0) as m:
        ids, _ = m.generate(prompt, 5)
        eos = int(ids[0, 1])
        ids2, lg2 = m.generate(prompt, 5, eos_id=eos)
    stop = int(np.argmax(ids2[0] == eos))
    assert stop <= 1
    assert np.all(ids2[0, stop + 1:] == -1) and np.all(lg2[0, stop + 1:] == 0)
    assert np.array_equal(ids2[0, :stop + 1], ids[0, :stop + 1])


@pytest.mark.gpu
def test_decoder_rejects_bad_arguments():
    pkg = load_pkg()
    w = _weights()
    with _decoder(w, 2, 128, 1, max_batch=2, max_seq=24) as m:
        with pytest.raises(pkg.MoeError):
            m.decode_step(np.zeros(2, np.int32))                     # before any prefill
        with pytest.raises(pkg.MoeError):
            m.prefill(pkg.synthetic_prompt(1, 3, 8, w.vocab))       # B > max_batch
        with pytest.raises(pkg.MoeError):
            m.generate(pkg.synthetic_prompt(1, 1, 20, w.vocab), 6)  # 20 + 6 - 1 > 24
        bad = np.array([[1, 2, w.vocab]], np.int32)
        with pytest.raises(pkg.MoeError) as ei:
            m.prefill(bad)                                           # id out of range
        assert "vocab" in str(ei.value)
        with pytest.raises(pkg.MoeError):
            m.decode_step(np.zeros(1, np.int32))                     # the failed prefill left no batch
        m.prefill(pkg.synthetic_prompt(1, 2, 8, w.vocab))
        with pytest.raises(ValueError):
            m.decode_step(np.zeros(3, np.int32))                     # not the prefill's batch
        # the decoder still works after the rejected calls
        lg, _ = m.prefill(pkg.synthetic_prompt(1, 2, 8, w.vocab))
        assert np.all(np.isfinite(lg))


@pytest.mark.gpu
def test_decoder_generate_reuses_and_recaptures_the_step_graph():
    """generate captures its decode step as a CUDA graph per (batch, eos,
    logits buffer, length): calls that change batch or length re-capture,
    a repeated call replays; each must still match the oracle."""
    pkg = load_pkg()
    w = _weights()
    o = _oracle(w, 2, 128)
    p3 = pkg.synthetic_prompt(8, 3, 12, w.vocab)
    p1 = p3[:1]
    with _decoder(w, 2, 128, 0) as m:
        runs = [(p3, 4), (p1, 5), (p1, 5), (p3, 4)]
        for prompt, n in runs:
            ids, lg = m.generate(prompt, n)
            ids_ref, lg_ref = o.generate(prompt, n)
            _check_greedy(ids, lg, ids_ref, lg_ref, 0)
        ids_nl, lg_nl = m.generate(p1, 5, want_logits=False)
        assert lg_nl is None
        ids_l, _ = m.generate(p1, 5)
        assert np.array_equal(ids_nl, ids_l)


def test_decoder_config_is_validated_before_any_device_work():
    """moe_decoder_create rejects shapes it cannot run before it looks at the
    weights or a device (no GPU needed)."""
    import ctypes
    pkg = load_pkg()
    L = pkg.load_library()
    bad = [(dict(head_dim=96), -2, "head_dim"),
           (dict(n_heads=3), -2, "n_heads"),
           (dict(vocab=250), -2, "vocab"),
           (dict(max_batch=0), -1, "max_batch"),
           (dict(precision=7), -1, "precision")]
    for kw, code, word in bad:
        cfg = pkg.decoder_config(n_layers=1, d_model=128, n_heads=1, head_dim=128, vocab=256,
                                 num_experts=8, top_k=2, d_ff=128, max_batch=2, max_seq=16)
        for k, v in kw.items():
            setattr(cfg, k, v)
        h = ctypes.c_void_p()
        cw = pkg.MoeDecoderWeightsC()          # all null: never reached
        rc = L.moe_decoder_create(ctypes.byref(cfg), ctypes.byref(cw), ctypes.byref(h))
        assert rc == code, (kw, rc)
        assert word in L.moe_last_error().decode()
        assert not h.value


@pytest.fixture(scope="module")
def config4_case():
    """Config-4 layer shapes, 2 layers: weights (drawn once, ~40 s on the host)
    and the oracle's prefill logits and 3 greedy tokens for 2 prompts of 64."""
    pkg = load_pkg()
    w = _weights(seed=4, n_layers=2, d=2048, vocab=32000, E=16, ff=5632)
    o = _oracle(w, 16, 128)
    prompt = pkg.synthetic_prompt(8, 2, 64, w.vocab)
    ids_ref, lg_ref = o.generate(prompt, 3)
    return w, prompt, ids_ref, lg_ref


@pytest.mark.gpu
@pytest.mark.parametrize("precision", [0, 1], ids=["fp32", "bf16"])
def test_decoder_at_config4_shapes(config4_case, precision):
    """The decoder at BASELINE config 4's layer shapes -- d 2048, 16 heads of
    128, 16 experts top-2 with d_ff 5632, vocabulary 32000 -- for 2 layers:
    prefill logits and 3 greedy tokens of 2 sequences of 64 against the
    oracle, within the same bounds as the small shape."""
    w, prompt, ids_ref, lg_ref = config4_case
    with _decoder(w, 16, 128, precision, max_batch=2, max_seq=80) as m:
        lg, _ = m.prefill(prompt)
        ids, lgg = m.generate(prompt, 3)
    assert rel_l2(lg, lg_ref[:, 0]) <= TOL[precision], rel_l2(lg, lg_ref[:, 0])
    _check_greedy(ids, lgg, ids_ref, lg_ref, precision)


# ---------------------------------------------------------------- fused batch-1 step
@pytest.mark.gpu
@pytest.mark.parametrize("heads,hd", [(2, 128), (4, 64)], ids=["hd128", "hd64"])
def test_fused_batch1_step_is_bit_identical_to_the_kernel_chain(heads, hd):
    """One sequence in BF16: with the fused step enabled the decode steps run
    as one cooperative launch; the kernel chain (the default) must give the
    same ids and bit-identical logits (every phase evaluates the chain's expressions in
    the chain's order), and both follow the oracle."""
    pkg = load_pkg()
    w = _weights()
    o = _oracle(w, heads, hd)
    prompt = pkg.synthetic_prompt(11, 1, 30, w.vocab)
    ids_ref, lg_ref = o.generate(prompt, 8)
    with _decoder(w, heads, hd, 1) as m:
        assert not m.fused_step_active
        m.set_fused_step(True)
        assert m.fused_step_active
        ids_f, lg_f = m.generate(prompt, 8)
        m.set_fused_step(False)
        assert not m.fused_step_active
        ids_c, lg_c = m.generate(prompt, 8)
        m.set_fused_step(True)
        ids_f2, lg_f2 = m.generate(prompt, 8)
    assert np.array_equal(ids_f, ids_c)
    assert np.array_equal(lg_f, lg_c)
    assert np.array_equal(lg_f2, lg_f)
    _check_greedy(ids_f, lg_f, ids_ref, lg_ref, 1)


@pytest.mark.gpu
def test_fused_step_serves_the_step_api_and_is_refused_in_fp32():
    pkg = load_pkg()
    w = _weights()
    prompt = pkg.synthetic_prompt(12, 1, 20, w.vocab)
    with _decoder(w, 2, 128, 1) as m:
        m.set_fused_step(True)
        ids, lg = m.generate(prompt, 4)
        l0, n0 = m.prefill(prompt)
        steps = [(l0, n0)]
        for _ in range(3):
            steps.append(m.decode_step(steps[-1][1]))
    for t, (lt, nt) in enumerate(steps):
        assert np.array_equal(lt, lg[:, t])
        assert np.array_equal(nt, ids[:, t])
    with _decoder(w, 2, 128, 0) as m:
        assert not m.fused_step_active
        with pytest.raises(pkg.MoeError) as ei:
            m.set_fused_step(True)
        assert "BF16" in str(ei.value)
        m.set_fused_step(False)


@pytest.mark.gpu
def test_fused_batch1_step_at_config4_shapes(config4_case):
    """Config-4 layer shapes (d 2048, 16 heads, 16 experts of 5632, vocab
    32000), 2 layers, one sequence: the fused step against the kernel chain
    (bit-identical) and against the oracle.  The prompt has 72 tokens: a
    prefill of at most 64 rows splits the projections' K with atomic adds,
    which would make the two runs' KV caches differ in the last bits."""
    pkg = load_pkg()
    w = config4_case[0]
    prompt = pkg.synthetic_prompt(13, 1, 72, w.vocab)
    ids_ref, lg_ref = _oracle(w, 16, 128).generate(prompt, 3)
    with _decoder(w, 16, 128, 1, max_batch=1, max_seq=80) as m:
        m.set_fused_step(True)
        ids_f, lg_f = m.generate(prompt, 3)
        m.set_fused_step(False)
        ids_c, lg_c = m.generate(prompt, 3)
    assert np.array_equal(ids_f, ids_c)
    assert np.array_equal(lg_f, lg_c)
    _check_greedy(ids_f, lg_f, ids_ref, lg_ref, 1)
