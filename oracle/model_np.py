"""Numpy FP32 restatement of the reference's native decode path.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): the checker for the CUDA
path and the timed CPU baseline, never part of the product.

Every function cites the reference code it restates.  ``HF:qwen3:<line>`` is
transformers' models/qwen3/modeling_qwen3.py (5.5.0 installed; the reference
pins 4.57.3, whose Qwen3 decoder arithmetic is the same).

The structure follows the native path: each CFG branch (cond, uncond) keeps
its own KV cache and runs its own prefill and trunk steps at positions
0..L-1 (model.py:623-676); the depth head is evaluated per branch
(model.py:573-578).  All arithmetic is float32; numpy's matmul goes to BLAS
sgemm/sgemv with float32 accumulation.
"""

from __future__ import annotations

import numpy as np

from . import sampler as _sampler

F32 = np.float32
DEPTH_NORM_EPS = float(np.finfo(np.float32).eps)  # nn.RMSNorm() default, model.py:135,137


def _np(t) -> np.ndarray:
    if isinstance(t, np.ndarray):
        return np.ascontiguousarray(t, dtype=F32)
    return np.ascontiguousarray(t.detach().cpu().numpy(), dtype=F32)


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """x * rsqrt(mean(x^2) + eps) * w  (HF:qwen3:59-64; torch nn.RMSNorm)."""
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=F32)
    inv = (F32(1.0) / np.sqrt(var + F32(eps))).astype(F32)
    return ((x * inv).astype(F32) * w).astype(F32)


def silu(g: np.ndarray) -> np.ndarray:
    """F.silu(g) = g * sigmoid(g)  (model.py:90, HF:qwen3:82)."""
    return (g / (F32(1.0) + np.exp(-g))).astype(F32)


def rope_tables(inv_freq: np.ndarray, positions: np.ndarray):
    """cos/sin [P, hd] as HF builds them (HF:qwen3:130-146): fp32 angle =
    inv_freq * position, duplicated over both halves; cos/sin of that fp32
    angle, correctly rounded back to fp32."""
    ang = (positions.astype(F32)[:, None] * inv_freq.astype(F32)[None, :]).astype(F32)
    emb = np.concatenate([ang, ang], axis=-1)
    return np.cos(emb.astype(np.float64)).astype(F32), np.sin(emb.astype(np.float64)).astype(F32)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """x*cos + rotate_half(x)*sin, neox style (HF:qwen3:151-181).
    x: [..., P, hd], cos/sin: [P, hd]."""
    h = x.shape[-1] // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
    return (x * cos + rot * sin).astype(F32)


class OracleModel:
    """Weights + the native path's functions, in numpy."""

    def __init__(self, state_dict, dims, inv_freq):
        self.dims = dims
        t, s = dims.trunk, dims.soraku
        self.cfg = s
        self.tcfg = t
        self.d = t.hidden_size
        self.H, self.KVH, self.hd = t.num_attention_heads, t.num_key_value_heads, t.head_dim
        self.n_rep = self.H // self.KVH
        self.eps = float(t.rms_norm_eps)
        self.scaling = float(self.hd ** -0.5)  # HF:qwen3:232
        self.inv_freq = _np(inv_freq)
        sd = {k: _np(v) for k, v in state_dict.items()}
        self.sd = sd
        self.layers = []
        for i in range(t.num_hidden_layers):
            p = f"trunk.layers.{i}."
            self.layers.append({
                "wq": sd[p + "self_attn.q_proj.weight"], "wk": sd[p + "self_attn.k_proj.weight"],
                "wv": sd[p + "self_attn.v_proj.weight"], "wo": sd[p + "self_attn.o_proj.weight"],
                "qn": sd[p + "self_attn.q_norm.weight"], "kn": sd[p + "self_attn.k_norm.weight"],
                "wg": sd[p + "mlp.gate_proj.weight"], "wu": sd[p + "mlp.up_proj.weight"],
                "wd": sd[p + "mlp.down_proj.weight"],
                "ln1": sd[p + "input_layernorm.weight"], "ln2": sd[p + "post_attention_layernorm.weight"],
            })
        self.final_norm = sd["trunk.norm.weight"]
        self.embed = sd["trunk.embed_tokens.weight"]
        self.table = sd["audio_codebooks.table"]
        self.scale = F32(s.num_codebooks ** -0.5)  # model.py:99
        self.depth = {
            "norm_in": sd["depth_head.norm_in.weight"], "norm_out": sd["depth_head.norm_out.weight"],
            "wg": sd["depth_head.mlp.gate_proj.weight"], "wu": sd["depth_head.mlp.up_proj.weight"],
            "wd": sd["depth_head.mlp.down_proj.weight"], "bias": sd["depth_head.bias"],
        }
        self.lang = sd.get("language_embeddings.weight")
        self.spk_proj = sd.get("speaker_projection.weight")
        self.spk_slot = sd.get("speaker_slot_embedding")

    # ------------------------------------------------------------ embeddings
    def frame_embedding(self, codes: np.ndarray) -> np.ndarray:
        """[..., Q] -> [..., d]: sum over q in order, then * scale (model.py:105-114)."""
        total = None
        for q in range(self.cfg.num_codebooks):
            piece = self.table[q][codes[..., q]]
            total = piece if total is None else (total + piece).astype(F32)
        return (total * self.scale).astype(F32)

    def embed_text(self, ids: np.ndarray) -> np.ndarray:
        """Text-table gather with language-ID substitution (model.py:326-338)."""
        ids = np.asarray(ids, dtype=np.int64)
        if not self.cfg.language_token_ids:
            return self.embed[ids]
        special = np.zeros(ids.shape, dtype=bool)
        index = np.zeros(ids.shape, dtype=np.int64)
        for j, ident in enumerate(self.cfg.language_token_ids):
            match = ids == ident
            special |= match
            index = np.where(match, j, index)
        ordinary = self.embed[np.where(special, 0, ids)]
        language = self.lang[index]
        return np.where(special[..., None], language, ordinary).astype(F32)

    def project_speaker(self, v) -> np.ndarray | None:
        """Linear(normalize(v)) (model.py:404-421); v: [192]."""
        if v is None:
            return None
        v = np.asarray(v, dtype=F32).reshape(-1)
        n = max(float(np.sqrt(np.sum(v.astype(np.float64) ** 2))), 1e-12)
        v = (v / F32(n)).astype(F32)
        return (self.spk_proj @ v).astype(F32)

    def start_embeds(self, ids, prompt_codes, speaker=None) -> np.ndarray:
        """[text][slot?][audio-BOS][prompt frames] (model.py:623-653)."""
        Q = self.cfg.num_codebooks
        text = self.embed_text(np.asarray(ids).reshape(-1))
        audio = np.full((1, Q), self.cfg.audio_bos_id, dtype=np.int64)
        if prompt_codes is not None and np.asarray(prompt_codes).size:
            audio = np.concatenate([audio, np.asarray(prompt_codes, dtype=np.int64).reshape(-1, Q)], 0)
        audio_e = self.frame_embedding(audio)
        parts = [text]
        spk = self.project_speaker(speaker)
        if spk is not None and self.cfg.speaker_condition_mode == "slot":
            parts.append((spk + self.spk_slot).astype(F32)[None])
        elif spk is not None:
            audio_e = audio_e.copy()
            audio_e[0] = (audio_e[0] + spk).astype(F32)
        parts.append(audio_e)
        return np.concatenate(parts, 0).astype(F32)

    # ----------------------------------------------------------------- trunk
    def _attn(self, layer, x, pos0, cache):
        """Self-attention block for x [L, d] at positions pos0..pos0+L-1 of one
        branch, appending to cache (HF:qwen3:240-291 with repeat_kv :184-193)."""
        L = x.shape[0]
        H, KVH, hd = self.H, self.KVH, self.hd
        n = rmsnorm(x, layer["ln1"], self.eps)
        q = (n @ layer["wq"].T).astype(F32).reshape(L, H, hd)
        k = (n @ layer["wk"].T).astype(F32).reshape(L, KVH, hd)
        v = (n @ layer["wv"].T).astype(F32).reshape(L, KVH, hd)
        q = rmsnorm(q, layer["qn"], self.eps).transpose(1, 0, 2)  # [H, L, hd]
        k = rmsnorm(k, layer["kn"], self.eps).transpose(1, 0, 2)
        v = v.transpose(1, 0, 2)
        cos, sin = rope_tables(self.inv_freq, np.arange(pos0, pos0 + L))
        q = apply_rope(q, cos, sin)
        k = apply_rope(k, cos, sin)
        if cache["k"] is None:
            cache["k"], cache["v"] = k, v
        else:
            cache["k"] = np.concatenate([cache["k"], k], axis=1)
            cache["v"] = np.concatenate([cache["v"], v], axis=1)
        K, Vv = cache["k"], cache["v"]
        T = K.shape[1]
        out = np.empty((H, L, hd), dtype=F32)
        qpos = np.arange(pos0, pos0 + L)
        kpos = np.arange(T)
        mask = kpos[None, :] > qpos[:, None]
        for h in range(H):
            j = h // self.n_rep
            s = (q[h] @ K[j].T).astype(F32) * F32(self.scaling)
            s = np.where(mask, -np.inf, s).astype(F32)
            m = s.max(axis=-1, keepdims=True)
            p = np.exp(s - m).astype(F32)
            p = (p / p.sum(axis=-1, keepdims=True, dtype=F32)).astype(F32)
            out[h] = (p @ Vv[j]).astype(F32)
        attn = out.transpose(1, 0, 2).reshape(L, H * hd)
        return (attn @ layer["wo"].T).astype(F32)

    def _mlp(self, layer, x):
        """x + down(silu(gate(n)) * up(n)), n = RMSNorm(x) (HF:qwen3:70-83,315-334)."""
        n = rmsnorm(x, layer["ln2"], self.eps)
        g = (n @ layer["wg"].T).astype(F32)
        u = (n @ layer["wu"].T).astype(F32)
        return ((silu(g) * u).astype(F32) @ layer["wd"].T).astype(F32)

    def new_cache(self):
        return {"layers": [{"k": None, "v": None} for _ in self.layers], "offset": 0}

    def run(self, cache, embeds: np.ndarray) -> np.ndarray:
        """Trunk over embeds [L, d] continuing at cache['offset'] (model.py:658-671,
        HF:qwen3:378-439).  Returns the final-normed hidden states [L, d]."""
        x = np.asarray(embeds, dtype=F32)
        pos0 = cache["offset"]
        for layer, lc in zip(self.layers, cache["layers"]):
            x = (x + self._attn(layer, x, pos0, lc)).astype(F32)
            x = (x + self._mlp(layer, x)).astype(F32)
        cache["offset"] += x.shape[0]
        return rmsnorm(x, self.final_norm, self.eps)

    # ------------------------------------------------------------ depth head
    def depth_body(self, x: np.ndarray) -> np.ndarray:
        """norm_out(a + mlp(a)), a = norm_in(x) (model.py:147-149)."""
        dp = self.depth
        a = rmsnorm(x, dp["norm_in"], DEPTH_NORM_EPS)
        g = (a @ dp["wg"].T).astype(F32)
        u = (a @ dp["wu"].T).astype(F32)
        y = (a + ((silu(g) * u).astype(F32) @ dp["wd"].T).astype(F32)).astype(F32)
        return rmsnorm(y, dp["norm_out"], DEPTH_NORM_EPS)

    def depth_step(self, hidden, prefix, q: int) -> np.ndarray:
        """body(hidden + prefix) @ table[q]^T + bias[q] (model.py:163-174)."""
        body = self.depth_body((hidden + prefix).astype(F32))
        return ((body @ self.table[q].T).astype(F32) + self.depth["bias"][q]).astype(F32)

    # --------------------------------------------------------------- loop
    def start(self, ids, prompt_codes, speaker=None):
        """Prefill of one branch (model.py:623-656); returns (cache, hidden[d])."""
        cache = self.new_cache()
        h = self.run(cache, self.start_embeds(ids, prompt_codes, speaker))
        return cache, h[-1].copy()

    def advance(self, cache, codes16) -> np.ndarray:
        """One trunk step on the frame's embedding (model.py:673-676)."""
        e = self.frame_embedding(np.asarray(codes16, dtype=np.int64).reshape(1, -1))
        return self.run(cache, e)[-1].copy()

    def teacher_forced(self, *, input_ids, uncond_input_ids, prompt_codes, codes, cfg_scale,
                       speaker=None, record_q=None):
        """Per-(frame, q) cond/uncond logits with the given codes fed back
        (the loop of model.py:567-612 with the draw replaced by the given code).

        Returns dict with 'hidden' [F, B, d] (hidden entering each frame),
        'logits' [F, nq, B, V] for q in record_q, 'merged' [F, nq, V]."""
        Q = self.cfg.num_codebooks
        record_q = list(range(Q)) if record_q is None else list(record_q)
        branches = [input_ids] + ([uncond_input_ids] if cfg_scale != 1.0 else [])
        states = [self.start(ids, prompt_codes, speaker) for ids in branches]
        caches = [s[0] for s in states]
        hiddens = [s[1] for s in states]
        codes = np.asarray(codes, dtype=np.int64).reshape(-1, Q)
        H, L, M = [], [], []
        for f in range(codes.shape[0]):
            H.append(np.stack(hiddens))
            prefix = np.zeros(self.d, dtype=F32)
            fl, fm = [], []
            for q in range(Q):
                if q in record_q:
                    lg = [self.depth_step(h, prefix, q) for h in hiddens]
                    fl.append(np.stack(lg))
                    if len(lg) > 1:
                        fm.append((lg[1] + F32(cfg_scale) * (lg[0] - lg[1])).astype(F32))
                    else:
                        fm.append(lg[0])
                prefix = (prefix + (self.table[q][codes[f, q]] * self.scale).astype(F32)).astype(F32)
            L.append(np.stack(fl))
            M.append(np.stack(fm))
            hiddens = [self.advance(c, codes[f]) for c in caches]
        return {"hidden": np.stack(H), "logits": np.stack(L), "merged": np.stack(M),
                "hidden_after": np.stack(hiddens)}

    def generate(self, *, input_ids, prompt_codes=None, max_new_frames=384, min_new_frames=4,
                 temperature=0.9, top_k=50, top_p=0.95, temperature_q0=None, top_k_q0=None,
                 top_p_q0=None, cfg_scale=1.0, uncond_input_ids=None, seed=0, request=0,
                 speaker=None, on_step=None, timings=None):
        """The native rollout (model.py:515-621) with the draw restated by
        oracle/sampler.c on Philox uniforms counter=(q, frame, request).
        ``timings`` (a dict) receives prefill_s and decode_s when given."""
        import time

        cfg = self.cfg
        Q = cfg.num_codebooks
        branches = [input_ids] + ([uncond_input_ids] if cfg_scale != 1.0 else [])
        t0 = time.perf_counter()
        states = [self.start(ids, prompt_codes, speaker) for ids in branches]
        t1 = time.perf_counter()
        caches = [s[0] for s in states]
        hiddens = [s[1] for s in states]
        frames = []
        stop = "max_frames"
        for index in range(max_new_frames):
            prefix = np.zeros(self.d, dtype=F32)
            row = []
            eos = False
            for q in range(Q):
                lg = [self.depth_step(h, prefix, q) for h in hiddens]
                t = temperature_q0 if q == 0 and temperature_q0 is not None else temperature
                k = top_k_q0 if q == 0 and top_k_q0 is not None else top_k
                p = top_p_q0 if q == 0 and top_p_q0 is not None else top_p
                u = _sampler.uniform(seed, request, index, q)
                code = _sampler.sample(
                    lg[0], lg[1] if len(lg) > 1 else None, cfg=cfg_scale, temperature=t,
                    top_k=k, top_p=p, mask_eos=(q != 0 or index < min_new_frames),
                    bos=cfg.audio_bos_id, pad=cfg.audio_pad_id, eos=cfg.audio_eos_id, u=u)
                if on_step is not None:
                    on_step(index, q, lg, code)
                if q == 0 and code == cfg.audio_eos_id:
                    eos = True
                    break
                row.append(code)
                prefix = (prefix + (self.table[q][code] * self.scale).astype(F32)).astype(F32)
            if eos:
                stop = "eos"
                break
            frames.append(row)
            hiddens = [self.advance(c, row) for c in caches]
        if timings is not None:
            timings["prefill_s"] = t1 - t0
            timings["decode_s"] = time.perf_counter() - t1
        codes = np.asarray(frames, dtype=np.int64).reshape(-1, Q)
        return codes, {"stop_reason": stop, "num_frames": codes.shape[0], "cfg_scale": cfg_scale}
