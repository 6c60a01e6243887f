"""Batched decode through swl_step_batch: several sequences advance together
through the batched kernels (one weight stream for all of them, grouped
routed experts). Checked against the CPU oracle (QwenCPUModel restatement) on
the tiny baseline model and on 4-layer 35B / 80B-shaped synthetic checkpoints,
and against the single-sequence path, within the north-star tolerances
(2e-2 max-abs, 1e-3 relative-L2 on logits; greedy tokens identical)."""
import ctypes as C

import numpy as np
import pytest

import oracle
import swiftlet_b200 as swl
from conftest import REF_FIXTURES, TINY_BASELINE
from swiftlet_b200 import formats
from swiftlet_b200.configs import NEXT_80B, Q35_35B, with_layers

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2 = 2e-2, 1e-3
# Inputs whose router comes closer than this to a top-k tie (relative gap
# between the k-th and (k+1)-th probability, measured in the oracle) are
# resampled: the router logits carry ~1e-6 of float summation-order noise in
# any implementation, so a nearer tie may legitimately route another expert.
ROUTE_GAP_MIN = 1e-5


def untied_prompt(cpu, V, n, seed, decode_steps):
    """A seeded length-`n` prompt whose oracle prefill and `decode_steps`
    greedy steps stay ROUTE_GAP_MIN away from every router top-k tie; returns
    the prompt, the oracle's logits after it and after each decode step, and
    the greedy tokens fed."""
    for attempt in range(8):
        rng = np.random.default_rng(seed + 7919 * attempt)
        prompt = rng.integers(0, V, n).tolist()
        cs = oracle.DecodeState()
        cpu.route_gap(reset=True)
        logits = [cpu.step(prompt, cs)]
        toks = []
        for _ in range(decode_steps):
            toks.append(int(np.argmax(logits[-1])))
            logits.append(cpu.step([toks[-1]], cs))
        if cpu.route_gap() >= ROUTE_GAP_MIN:
            return prompt, logits, toks
    pytest.fail(f"no prompt of length {n} without a router near-tie in 8 draws")


def stepwise(gpu, tokens, state):
    """Logits after feeding `tokens` one at a time through the single-token
    decode kernels (the reference for chunked steps)."""
    for t in tokens:
        lg = gpu.step([t], state)
    return lg


def assert_close(got, ref, what):
    err = float(np.abs(got - ref).max())
    rel = float(np.linalg.norm(got - ref) / (np.linalg.norm(ref) + 1e-30))
    assert err < MAX_ABS and rel < REL_L2, f"{what}: max-abs {err:.3e}, rel-L2 {rel:.3e}"


def test_tiny_baseline_ragged_batch_matches_oracle():
    gpu = swl.QwenCUDAModel(TINY_BASELINE)
    cpu = oracle.OracleModel(TINY_BASELINE)
    ok, why = gpu.batch_supported()
    assert ok, why
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, 256, n).tolist() for n in (1, 5, 9, 3, 12)]
    gs = [gpu.new_state(64) for _ in prompts]
    cs = [oracle.DecodeState() for _ in prompts]
    gl = gpu.step_batch(prompts, gs)
    for i, p in enumerate(prompts):
        assert gs[i].position == len(p)
        assert_close(gl[i], cpu.step(p, cs[i]), f"prompt {i}")
    toks = [int(np.argmax(r)) for r in gl]
    for step in range(8):
        gl = gpu.step_batch([[t] for t in toks], gs)
        nxt = []
        for i in range(len(prompts)):
            cl = cpu.step([toks[i]], cs[i])
            assert_close(gl[i], cl, f"step {step} seq {i}")
            assert int(np.argmax(gl[i])) == int(np.argmax(cl)), (step, i)
            nxt.append(int(np.argmax(gl[i])))
        toks = nxt
    gpu.close()


@pytest.fixture(scope="module", params=["35b", "80b"])
def synth(request, tmp_path_factory):
    shape = {"35b": Q35_35B, "80b": NEXT_80B}[request.param]
    d = formats.write_synthetic(str(tmp_path_factory.mktemp("bsyn") / request.param), with_layers(shape, 4), seed=99)
    gpu = swl.QwenCUDAModel(d)
    yield request.param, d, gpu
    gpu.close()


def test_synthetic_batch_matches_oracle(synth):
    _, d, gpu = synth
    assert gpu.batch_supported()[0]
    cpu = oracle.OracleModel(d, retain_all_layers=True)
    V = gpu.config.vocab_size
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, V, n).tolist() for n in (2, 1, 3)]
    gs = [gpu.new_state(32) for _ in prompts]
    cs = [oracle.DecodeState() for _ in prompts]
    gl = gpu.step_batch(prompts, gs)
    for i, p in enumerate(prompts):
        assert_close(gl[i], cpu.step(p, cs[i]), f"prompt {i}")
    toks = [int(np.argmax(r)) for r in gl]
    for step in range(2):
        gl = gpu.step_batch([[t] for t in toks], gs)
        for i in range(len(prompts)):
            cl = cpu.step([toks[i]], cs[i])
            assert_close(gl[i], cl, f"step {step} seq {i}")
            assert int(np.argmax(gl[i])) == int(np.argmax(cl))
        toks = [int(np.argmax(r)) for r in gl]


@pytest.mark.parametrize("nseq", [16, 64, 70])
def test_full_batch_matches_single_sequence_path(synth, nseq):
    """nseq sequences at ragged positions: the batched logits equal the
    single-sequence kernels' (themselves checked against the oracle) within
    the tolerances; 70 sequences take two launches (64 + 6)."""
    _, _, gpu = synth
    V = gpu.config.vocab_size
    rng = np.random.default_rng(nseq)
    prompts = [rng.integers(0, V, int(rng.integers(1, 5))).tolist() for _ in range(nseq)]
    bs = [gpu.new_state(16) for _ in range(nseq)]
    ss = [gpu.new_state(16) for _ in range(nseq)]
    bl = gpu.step_batch(prompts, bs)
    for i, p in enumerate(prompts):
        assert_close(bl[i], stepwise(gpu, p, ss[i]), f"prompt {i}")
    toks = rng.integers(0, V, nseq).tolist()
    bl = gpu.step_batch([[t] for t in toks], bs)
    for i in range(nseq):
        assert_close(bl[i], gpu.step([toks[i]], ss[i]), f"decode {i}")
    for s in bs + ss:
        s.free()


def test_long_context_batch_matches_single_sequence_path(synth):
    """Contexts past several attention chunk clusters (ragged 150..300
    positions) through the batched rounds."""
    _, _, gpu = synth
    V = gpu.config.vocab_size
    rng = np.random.default_rng(11)
    prompts = [rng.integers(0, V, n).tolist() for n in (300, 150, 231)]
    bs = [gpu.new_state(512) for _ in prompts]
    ss = [gpu.new_state(512) for _ in prompts]
    bl = gpu.step_batch(prompts, bs)
    for i, p in enumerate(prompts):
        assert_close(bl[i], stepwise(gpu, p, ss[i]), f"prompt {i}")
    # decode continues from the chunked contexts
    toks = [int(np.argmax(r)) for r in bl]
    bl = gpu.step_batch([[t] for t in toks], bs)
    for i in range(len(prompts)):
        assert_close(bl[i], gpu.step([toks[i]], ss[i]), f"decode {i}")
    for s in bs + ss:
        s.free()


@pytest.mark.parametrize("n", [2, 63, 64, 65, 130])
def test_chunked_prefill_matches_stepwise(synth, n):
    """A single sequence's prompt through swl_step runs in chunks of up to 64
    tokens (one weight stream per chunk; 16+ tokens per sequence take the
    chunk-parallel delta rule); it and feeding the tokens one at a time both
    match the CPU oracle after the prompt and for two decode steps from the
    states they leave."""
    _, d, gpu = synth
    cpu = oracle.OracleModel(d, retain_all_layers=True)
    prompt, ref, toks = untied_prompt(cpu, gpu.config.vocab_size, n, 1000 + n, 2)
    a, b = gpu.new_state(256), gpu.new_state(256)
    la = gpu.step(prompt, a)
    assert a.position == n
    assert_close(la, ref[0], f"chunked prefill {n}")
    assert_close(stepwise(gpu, prompt, b), ref[0], f"token-by-token prefill {n}")
    for step, t in enumerate(toks):
        la, lb = gpu.step([t], a), gpu.step([t], b)
        assert_close(la, ref[step + 1], f"decode {step} after chunked prefill {n}")
        assert_close(lb, ref[step + 1], f"decode {step} after token-by-token prefill {n}")
    a.free()
    b.free()


def test_device_batch_greedy_feedback(synth):
    """swl_step_batch_device with the greedy ids written over the token
    buffer gives the same tokens as host-side argmax of swl_step_batch."""
    torch = pytest.importorskip("torch")
    _, _, gpu = synth
    V = gpu.config.vocab_size
    n = 8
    rng = np.random.default_rng(5)
    toks = rng.integers(0, V, n).astype(np.int32)
    a = [gpu.new_state(16) for _ in range(n)]
    b = [gpu.new_state(16) for _ in range(n)]
    d_tok = torch.tensor(toks, dtype=torch.int32, device="cuda")
    host = toks.tolist()
    for _ in range(3):
        gpu.step_batch_device(a, d_tok.data_ptr(), 0, d_tok.data_ptr())
        host = [int(np.argmax(r)) for r in gpu.step_batch([[t] for t in host], b)]
        torch.cuda.synchronize()
        assert d_tok.cpu().tolist() == host
    for s in a + b:
        s.free()


def test_unsupported_formats_step_one_by_one():
    """The f32 reference fixture has plain weights: the batch runs the
    sequences one by one and still matches the oracle."""
    d = f"{REF_FIXTURES}/tiny-model"
    gpu = swl.QwenCUDAModel(d)
    ok, why = gpu.batch_supported()
    assert not ok and why
    cpu = oracle.OracleModel(d)
    prompts = [[1, 5, 9], [42]]
    gs = [gpu.new_state(16) for _ in prompts]
    cs = [oracle.DecodeState() for _ in prompts]
    gl = gpu.step_batch(prompts, gs)
    for i, p in enumerate(prompts):
        assert np.abs(gl[i] - cpu.step(p, cs[i])).max() < 2e-3
    gpu.close()


def test_batch_rejects_a_repeated_state():
    gpu = swl.QwenCUDAModel(TINY_BASELINE)
    s = gpu.new_state(16)
    handles = (C.c_void_p * 2)(s._bind(gpu), s._bind(gpu))
    toks = np.array([1, 2], np.int32)
    counts = np.array([1, 1], np.int32)
    out = np.empty((2, gpu.config.vocab_size), np.float32)
    rc = swl.lib().swl_step_batch(gpu._h, handles, toks.ctypes.data, counts.ctypes.data, 2, out.ctypes.data)
    assert rc == swl.SWL_ERR_INVALID
    gpu.close()
