"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a container where the reference checkout is importable:

    python tests/golden/make_golden.py --reference <path to soraku-TTS checkout>

It builds the reference's ``SorakuTTSv2`` (soraku_inference/model.py:177) on a
transformers Qwen3 trunk, loads the seeded random weights of
``soraku_tts_b200.weights.random_state_dict`` into it, and records:

* ``model_small.npz`` -- 2-layer trunk (text vocab 4096) with random norm
  gains and depth bias: per-(frame, q) cond/uncond logits and the hidden state
  entering each frame, teacher-forced on seeded codes through the reference's
  own ``_start_state`` / ``depth_head.step`` / ``_advance`` (model.py:561-612);
  plus the codes of the reference's greedy ``generate`` (temperature 0).
* ``model_route_d.npz`` -- the same with four language IDs and a slot-mode
  speaker vector (model.py:186-209, 326-338, 404-421, 644-648).
* ``model_full.npz`` -- the benchmark model (28 layers, vocab 151936, seed 42,
  unit norms, zero bias) on config 1's prompt shape (1 + 48 text ids, 72
  reference frames), two teacher-forced frames, q in {0, 15}.
* ``sampler_cases.npz`` -- merged logits through the native CFG/mask lines
  (model.py:579-584) and ``_sample_logits`` (model.py:686-708) with
  ``torch.multinomial`` intercepted, so each case stores the reference's final
  probability vector; greedy cases store the reference's argmax.

Weights are not stored: the seed and dimensions regenerate them anywhere.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from soraku_tts_b200.config import ModelDims, SorakuV2Config, TrunkConfig  # noqa: E402
from soraku_tts_b200.weights import random_state_dict  # noqa: E402


def build_reference(dims: ModelDims, sd):
    from transformers import AutoModel, Qwen3Config
    from soraku_inference.model import SorakuTTSv2
    from soraku_inference.model import SorakuV2Config as RefCfg

    trunk = AutoModel.from_config(Qwen3Config(**dims.trunk.to_hf_kwargs()), dtype=torch.float32,
                                  attn_implementation="sdpa")
    s = dims.soraku
    cfg = RefCfg(num_codebooks=s.num_codebooks, codebook_size=s.codebook_size,
                 depth_ffn_mult=s.depth_ffn_mult, speaker_conditioning=s.speaker_conditioning,
                 speaker_dim=s.speaker_dim, speaker_condition_mode=s.speaker_condition_mode,
                 language_token_ids=tuple(s.language_token_ids))
    model = SorakuTTSv2(cfg, trunk=trunk)
    missing, unexpected = model.load_state_dict(sd, strict=True)
    assert not missing and not unexpected
    return model.eval()


@torch.inference_mode()
def teacher_forced(model, ids, uncond, prompt, codes, cfg_scale, record_q, speaker=None):
    """The reference loop body (model.py:561-612) with the codes fed back."""
    import torch.nn.functional as F

    branches = [ids] + ([uncond] if cfg_scale != 1.0 else [])
    states = [model._start_state(b, prompt, speaker) for b in branches]
    table = model.audio_codebooks.table
    Q = model.config.num_codebooks
    H, L = [], []
    for f in range(codes.shape[0]):
        hiddens = [s["hidden"] for s in states]
        H.append(torch.cat(hiddens).numpy())
        prefix = [torch.zeros_like(hiddens[0]) for _ in states]
        fl = []
        for q in range(Q):
            if q in record_q:
                lg = [model.depth_head.step(hiddens[b], prefix[b], q, table)[0].float()
                      for b in range(len(states))]
                fl.append(torch.stack(lg).numpy())
            tok = torch.tensor([int(codes[f, q])])
            emb = F.embedding(tok, table[q]) * model.audio_codebooks.scale
            for b in range(len(states)):
                prefix[b] = prefix[b] + emb
        L.append(np.stack(fl))
        frame = torch.tensor(codes[f], dtype=torch.long).view(1, 1, -1)
        for s in states:
            s["hidden"] = model._advance(s, frame)
    after = torch.cat([s["hidden"] for s in states]).numpy()
    return np.stack(H), np.stack(L), after


def versions():
    import transformers
    return {"torch": torch.__version__, "transformers": transformers.__version__,
            "numpy": np.__version__}


def make_model_case(name, dims, *, seed, random_norms, random_bias, n_text, n_ref, n_frames,
                    record_q, language=None, speaker_seed=None, greedy_frames=0, ids_seed=1234):
    t0 = time.time()
    sd = random_state_dict(dims, seed, random_norms=random_norms, random_bias=random_bias)
    model = build_reference(dims, sd)
    s = dims.soraku
    rng = np.random.default_rng(ids_seed)
    bos_text = min(151643, dims.trunk.vocab_size - 6)
    text = rng.integers(0, bos_text, size=n_text).tolist()
    ids = [bos_text]
    if language is not None:
        ids.append(int(s.language_token_ids[language]))
    ids += text
    ids = torch.tensor([ids], dtype=torch.long)
    uncond = torch.tensor([[bos_text]], dtype=torch.long)
    prompt = torch.tensor(rng.integers(0, s.codebook_size, size=(n_ref, s.num_codebooks)),
                          dtype=torch.long)
    codes = rng.integers(0, s.codebook_size, size=(n_frames, s.num_codebooks)).astype(np.int64)
    speaker = None
    if speaker_seed is not None:
        g = torch.Generator().manual_seed(speaker_seed)
        v = torch.randn(1, s.speaker_dim, generator=g)
        speaker = v / v.norm(dim=-1, keepdim=True)
    cfg_scale = 1.5
    H, L, after = teacher_forced(model, ids, uncond, prompt, codes, cfg_scale, record_q, speaker)
    out = dict(input_ids=ids.numpy(), uncond_input_ids=uncond.numpy(), prompt_codes=prompt.numpy(),
               codes=codes, hidden=H.astype(np.float32), logits=L.astype(np.float32),
               hidden_after=after.astype(np.float32), record_q=np.array(record_q, dtype=np.int64))
    if speaker is not None:
        out["speaker"] = speaker.numpy().astype(np.float32)
    if greedy_frames:
        with torch.inference_mode():
            gcodes, info = model.generate(input_ids=ids, prompt_codes=prompt,
                                          max_new_frames=greedy_frames, min_new_frames=greedy_frames,
                                          temperature=0.0, cfg_scale=cfg_scale,
                                          uncond_input_ids=uncond, seed=7,
                                          speaker_embedding=speaker)
        out["greedy_codes"] = gcodes.numpy()
    meta = dict(name=name, seed=seed, random_norms=random_norms, random_bias=random_bias,
                cfg_scale=cfg_scale, trunk=dims.trunk.__dict__, soraku=dims.soraku.to_dict(),
                versions=versions())
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(f"{name}: {time.time() - t0:.1f}s")


def make_sampler_cases(n_random=64, seed=2024):
    from soraku_inference import model as refmodel

    captured = {}
    real_multinomial = torch.multinomial

    def spy(probs, num_samples, *a, **k):
        captured["p"] = probs.detach().clone()
        return real_multinomial(probs, num_samples, *a, **k)

    V, bos, eos, pad = 2051, 2048, 2049, 2050
    rng = np.random.default_rng(seed)
    rows = []
    specs = []
    for i in range(n_random):
        sigma = [0.5, 2.0, 5.0][i % 3]
        cond = rng.normal(0, sigma, V).astype(np.float32)
        uncond = (cond * 0.7 + rng.normal(0, sigma * 0.5, V)).astype(np.float32)
        cfg = [1.5, 1.0, 2.5][(i // 3) % 3]
        temp = [0.9, 0.5, 1.3, 0.0][(i // 9) % 4]
        top_k = [50, 1, None, 2051, 7][(i // 2) % 5]
        top_p = [0.95, 0.5, None, 1.0][(i // 5) % 4]
        mask_eos = bool(i % 2)
        if i % 11 == 0:  # ties at and around the top-k cutoff
            cond[:] = np.round(cond * 2) / 2
            uncond[:] = cond
        specs.append((cond, uncond, cfg, temp, top_k, top_p, mask_eos))
    torch.multinomial = spy
    try:
        for cond, uncond, cfg, temp, top_k, top_p, mask_eos in specs:
            c = torch.from_numpy(cond)
            u = torch.from_numpy(uncond)
            merged = c if cfg == 1.0 else u + cfg * (c - u)  # model.py:579-581
            blocked = torch.zeros(V, dtype=torch.bool)
            blocked[bos] = True
            blocked[pad] = True
            merged = merged.masked_fill(blocked, -torch.inf)  # model.py:582
            if mask_eos:
                merged[eos] = -torch.inf  # model.py:583-584
            captured.clear()
            code = refmodel._sample_logits(merged.clone(), temperature=temp, top_k=top_k,
                                           top_p=top_p, generator=torch.Generator().manual_seed(0))
            probs = captured["p"].numpy() if "p" in captured else np.full(V, np.nan, np.float32)
            rows.append(dict(cond=cond, uncond=uncond, cfg=cfg, temp=temp,
                             top_k=-1 if top_k is None else top_k,
                             top_p=-1.0 if top_p is None else top_p, mask_eos=mask_eos,
                             probs=probs, code=code))
    finally:
        torch.multinomial = real_multinomial
    out = {k: np.stack([np.asarray(r[k]) for r in rows]) for k in rows[0]}
    out["meta"] = np.array(json.dumps(dict(V=V, bos=bos, eos=eos, pad=pad, versions=versions())))
    np.savez_compressed(os.path.join(HERE, "sampler_cases.npz"), **out)
    print(f"sampler_cases: {len(rows)} cases")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    only = set(args.only.split(",")) if args.only else None

    def want(n):
        return only is None or n in only

    small_trunk = TrunkConfig(num_hidden_layers=2, vocab_size=4096)
    if want("sampler_cases"):
        make_sampler_cases()
    if want("model_small"):
        make_model_case("model_small", ModelDims(SorakuV2Config(), small_trunk), seed=11,
                        random_norms=True, random_bias=True, n_text=12, n_ref=6, n_frames=3,
                        record_q=[0, 1, 2, 7, 15], greedy_frames=3)
    if want("model_route_d"):
        s = SorakuV2Config(language_token_ids=(4091, 4092, 4093, 4094), speaker_conditioning=True,
                           speaker_condition_mode="slot")
        make_model_case("model_route_d", ModelDims(s, small_trunk), seed=5, random_norms=True,
                        random_bias=True, n_text=10, n_ref=5, n_frames=2, record_q=[0, 3, 15],
                        language=1, speaker_seed=7)
    if want("model_full"):
        make_model_case("model_full", ModelDims(), seed=42, random_norms=False, random_bias=False,
                        n_text=48, n_ref=72, n_frames=2, record_q=[0, 15], greedy_frames=0)
    if want("model_route_d_full"):
        # config 3 at benchmark size: 28 layers, four language IDs, slot-mode
        # speaker vector (seed 7), text and reference lengths drawn from
        # U[16, 96] and U[24, 144]
        rng = np.random.default_rng(3)
        n_text, n_ref = int(rng.integers(16, 97)), int(rng.integers(24, 145))
        s = SorakuV2Config(language_token_ids=(151669, 151670, 151671, 151672), speaker_conditioning=True,
                           speaker_condition_mode="slot")
        make_model_case("model_route_d_full", ModelDims(s), seed=42, random_norms=False, random_bias=False,
                        n_text=n_text, n_ref=n_ref, n_frames=2, record_q=[0, 15], language=2, speaker_seed=7,
                        ids_seed=77)
    if want("model_bos"):
        # speaker vector added to the audio-BOS frame (model.py:649-651)
        s = SorakuV2Config(speaker_conditioning=True, speaker_condition_mode="bos")
        make_model_case("model_bos", ModelDims(s, small_trunk), seed=9, random_norms=True,
                        random_bias=True, n_text=14, n_ref=7, n_frames=2, record_q=[0, 5, 15],
                        speaker_seed=8)


if __name__ == "__main__":
    main()
