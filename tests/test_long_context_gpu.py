"""Decode parity on the GPU at the benchmark's context lengths and batch shapes.

Every case is checked against the oracle (the reference's native FP32 path
restated in numpy, pinned to the reference by tests/golden) teacher-forced on
the engine's own codes:

* per-(frame, q) cond/uncond logits within rel/abs 1e-4 at the recorded
  codebooks (the oracle runs every frame's trunk step, so the context grows
  exactly as in the engine);
* every drawn code, at every (frame, q), bit-exact with the oracle's sampler
  fed the engine's logits and the same Philox uniform;
* top-50 sets of the merged logits agree on >= 99 % of the recorded steps.

Shapes: config 2 (1 + 96 text ids, 144 reference frames, 600 decoded frames:
context 242 -> 842 cond, 146 -> 746 uncond) on the 2-layer weights; prompts of
~1400 positions (several rounds of staged keys per attention CTA) on 2 and 28
layers; ragged multi-request batches drawn like config 4 (text U[16, 96],
reference U[24, 144], one seed and one random stream per request) at 16 rows
and at 64 requests (128 rows).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sampler as osamp
from tests._util import assert_close, load_golden, oracle_from_meta

pytestmark = pytest.mark.gpu
TOL = dict(rtol=1e-4, atol=1e-4)
BOS, EOS, PAD = 2048, 2049, 2050


def _setup(name):
    from soraku_tts_b200.model import SorakuModel

    data, meta = load_golden(name)
    orc, dims, sd = oracle_from_meta(meta)
    return orc, dims, SorakuModel(dims, sd, "cuda")


@pytest.fixture(scope="module")
def small():
    return _setup("model_small")


@pytest.fixture(scope="module")
def full():
    return _setup("model_full")


def _prompt(dims, seed, n_text, n_ref):
    rng = np.random.default_rng(seed)
    bos_text = min(151643, dims.trunk.vocab_size - 6)
    ids = np.concatenate([[bos_text], rng.integers(0, bos_text, n_text)]).astype(np.int64)
    uncond = np.array([bos_text], np.int64)
    prompt = rng.integers(0, 2048, size=(n_ref, 16)).astype(np.int64)
    return ids, uncond, prompt


def _decode_batch(model, prompts, n_frames, seeds, *, max_len, fpg=1):
    """Prefill every request, decode n_frames with the debug logits history.
    Returns codes [req][F, Q] and logits [F, Q, rows, V]."""
    from soraku_tts_b200.graph_frame import NativeEngine

    n = len(prompts)
    Q, V = model.config.num_codebooks, model.config.audio_vocab_size
    longest = max(len(p[0]) + len(p[2]) + 2 for p in prompts)
    eng = NativeEngine(model, max_requests=n, rows_per_request=2, max_len=max_len, max_frames=n_frames,
                       max_prefill=longest)
    eng.set_debug(True)
    for r, ((ids, unc, pc), seed) in enumerate(zip(prompts, seeds)):
        eng.set_sampling(r, cfg=1.5, temperature=0.9, temperature_q0=0.9, top_k=50, top_p=0.95, top_k_q0=50,
                         top_p_q0=0.95, seed=seed, min_new_frames=10 ** 6, eos_rule=1)
        eng.prefill(r, ids, unc, pc)
    eng.capture(n, fpg)
    logits = np.empty((n_frames, Q, 2 * n, V), np.float32)
    for f in range(n_frames):
        eng.step(True)
        torch.cuda.synchronize()
        logits[f] = eng.view(4).view(Q, 2 * n, V).cpu().numpy()
    codes = [eng.read_codes(r, 0, n_frames).clone().numpy() for r in range(n)]
    err = eng.view(6, torch.int32).cpu().numpy()
    assert (err == 0).all(), f"device error flags raised: {err}"
    eng.close()
    return codes, logits


def _check_request(orc, prompt, codes, logits, *, seed, stream, record_q, what):
    """logits: this request's [F, Q, 2, V]."""
    ids, unc, pc = prompt
    tf = orc.teacher_forced(input_ids=ids, uncond_input_ids=unc, prompt_codes=pc, codes=codes, cfg_scale=1.5,
                            record_q=record_q)
    assert_close(logits[:, record_q], tf["logits"], what=f"{what}: logits at q {record_q}", **TOL)
    F, Q = codes.shape
    for f in range(F):
        for q in range(Q):
            c, u = logits[f, q, 0], logits[f, q, 1]
            want = osamp.sample(c, u, cfg=1.5, temperature=0.9, top_k=50, top_p=0.95, mask_eos=True, bos=BOS,
                                pad=PAD, eos=EOS, u=osamp.uniform(seed, stream, f, q))
            assert int(codes[f, q]) == want, f"{what}: frame {f} q {q} drew {codes[f, q]}, oracle {want}"
    agree = total = 0
    for f in range(F):
        for j, q in enumerate(record_q):
            c, u = logits[f, q, 0], logits[f, q, 1]
            m_gpu = u + np.float32(1.5) * (c - u)
            m_orc = tf["merged"][f, j]
            top_gpu = set(np.argsort(-m_gpu)[:50].tolist())
            top_orc = set(np.argsort(-m_orc)[:50].tolist())
            agree += top_gpu == top_orc
            total += 1
    assert agree / total >= 0.99, f"{what}: top-50 agreement {agree}/{total}"


def test_config2_length_600_frames(small):
    """Config 2's prompt shape and all 600 frames (context to 842 positions)."""
    orc, dims, model = small
    prompt = _prompt(dims, 1000, 96, 144)
    codes, logits = _decode_batch(model, [prompt], 600, [71], max_len=1024)
    _check_request(orc, prompt, codes[0], logits[:, :, 0:2], seed=71, stream=0, record_q=[0, 15],
                   what="config-2 length")


def test_long_prompt_multi_round_attention_2layer(small):
    """~1400 cached positions: every attention CTA walks several rounds of keys."""
    orc, dims, model = small
    prompt = _prompt(dims, 5, 96, 1300)
    codes, logits = _decode_batch(model, [prompt], 12, [72], max_len=1536)
    _check_request(orc, prompt, codes[0], logits[:, :, 0:2], seed=72, stream=0, record_q=[0, 7, 15],
                   what="2-layer 1400-position context")


def test_long_prompt_multi_round_attention_28layer(full):
    """The 28-layer benchmark model at ~1400 cached positions."""
    orc, dims, model = full
    prompt = _prompt(dims, 6, 96, 1300)
    codes, logits = _decode_batch(model, [prompt], 4, [73], max_len=1536)
    _check_request(orc, prompt, codes[0], logits[:, :, 0:2], seed=73, stream=0, record_q=[0, 15],
                   what="28-layer 1400-position context")


def _ragged(dims, n, base_seed):
    rng = np.random.default_rng(base_seed)
    out = []
    for i in range(n):
        out.append(_prompt(dims, base_seed + 1 + i, int(rng.integers(16, 97)), int(rng.integers(24, 145))))
    return out


def test_ragged_requests_16_rows(small):
    """8 requests with their own text and reference lengths decoded as one
    16-row batch (the tensor-core GEMM and the double-buffered attention)."""
    orc, dims, model = small
    prompts = _ragged(dims, 8, 400)
    seeds = [500 + i for i in range(8)]
    codes, logits = _decode_batch(model, prompts, 4, seeds, max_len=512)
    for r in range(8):
        _check_request(orc, prompts[r], codes[r], logits[:, :, 2 * r:2 * r + 2], seed=seeds[r], stream=r,
                       record_q=[0, 7, 15], what=f"request {r}")


def test_ragged_requests_config4_shape(small):
    """64 requests drawn like config 4 (128 rows) on the 2-layer weights."""
    orc, dims, model = small
    prompts = _ragged(dims, 64, 900)
    seeds = [2000 + i for i in range(64)]
    codes, logits = _decode_batch(model, prompts, 2, seeds, max_len=512)
    for r in range(64):
        _check_request(orc, prompts[r], codes[r], logits[:, :, 2 * r:2 * r + 2], seed=seeds[r], stream=r,
                       record_q=[0, 15], what=f"request {r}")
