"""Oracle: the reference's dense decode layer and its greedy drivers (numpy).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates src/lumina_framework/chat.py and the tree verifier of eagle.py/spec.py
with the same numpy operations in the same order, so that on one machine the
results equal the reference's bit for bit (checked against golden vectors made
by the reference itself):

  * ``rmsnorm``         chat.py:63-66  (eps 1e-6, fp32)
  * ``rope_freqs``      chat.py:69-75  (fp32 angles, rotate-half layout)
  * ``rope_angles_at``  chat.py:78-85
  * ``apply_rope``      chat.py:88-103
  * ``OracleModel``     ChatModel.from_tensors (every tensor fp16-rounded,
    chat.py:138-143; head = lm_head or the tied embedding, :194-195) and
    ``_layer`` chat.py:232-304 (GQA repeat before caching :257-263, causal +
    tree bias :264-274, fp32 softmax attention :275-281, SwiGLU with the
    ±40 clip :300-304, virtual-MoE branch :285-299)
  * ``generate`` / ``generate_cached``  chat.py:307-407, 410-551 (greedy
    ``pick`` path; no final norm before the head, :388/:529)
  * ``pld_draft`` / ``generate_spec``  chat.py:553-648
  * ``build_tree_mask`` spec.py:56-83; ``verify_tree`` eagle.py:259-291;
    ``commit_verified`` eagle.py:294-357
  * ``moe_grouped_forward`` qwen_next.py:31-78 (unit weights)
"""
from __future__ import annotations

import numpy as np


def rmsnorm(x, w, eps=1e-6):
    xf = x.astype(np.float32)
    m = np.mean(xf ** 2, axis=-1, keepdims=True)
    return (xf / np.sqrt(m + eps) * w.astype(np.float32)).astype(np.float32)


def _freqs(head_dim, theta):
    return 1.0 / (theta ** (np.arange(0, 2 * (head_dim // 2), 2).astype(np.float32) / head_dim))


def rope_freqs(head_dim, seq_len, theta=1000000.0, offset=0):
    t = np.arange(offset, offset + seq_len, dtype=np.float32)
    angles = np.outer(t, _freqs(head_dim, theta))
    return np.concatenate([angles, angles], axis=-1)


def rope_angles_at(head_dim, positions, theta=1000000.0):
    angles = np.outer(np.asarray(positions, dtype=np.float32), _freqs(head_dim, theta))
    return np.concatenate([angles, angles], axis=-1)


def apply_rope(x, angles):
    P = angles.shape[-1] // 2
    xr, rest = x[..., :2 * P], x[..., 2 * P:]
    x1, x2 = xr[..., :P], xr[..., P:]
    a1, a2 = angles[..., :P], angles[..., P:]
    out = np.concatenate([x1 * np.cos(a1) - x2 * np.sin(a1),
                          x1 * np.sin(a2) + x2 * np.cos(a2)], axis=-1)
    if rest.shape[-1]:
        out = np.concatenate([out, rest], axis=-1)
    return out


def _sigmoid(x):
    """qwen_next.py:23-24 (clip to +-40, float32 exponent)."""
    return 1.0 / (1.0 + np.exp(-np.clip(x, -40, 40).astype(np.float32)))


def moe_grouped_forward(h, gate_up, down, router_w, top_k, router_b=None,
                        router_feat="raw"):
    """qwen_next.py:31-78 with gate_fn="sigmoid", weight_mode="unit"."""
    E = gate_up.shape[0]
    I = gate_up.shape[1] // 2
    rf = np.abs(h) if router_feat == "abs" else h
    logits = rf @ router_w.T
    if router_b is not None:
        logits = logits + np.asarray(router_b, dtype=np.float32)
    scores = _sigmoid(logits)
    k = max(1, min(top_k, E))
    idx = np.argsort(-scores, axis=1)[:, :k]
    out = np.zeros_like(h, dtype=np.float32)
    for s in range(h.shape[0]):
        acc = np.zeros(h.shape[1], dtype=np.float32)
        for j in range(k):
            e = int(idx[s, j])
            gu = gate_up[e] @ h[s]
            g, u = gu[:I], gu[I:]
            silu = g / (1.0 + np.exp(-np.clip(g, -40, 40)))
            acc += 1.0 * (down[e].T @ (silu * u))
        out[s] = acc
    return out.astype(np.float32), {"experts": idx}


class OracleModel:
    """ChatModel built from a tensor dict (chat.py:128-222), fast=False."""

    def __init__(self, tensors: dict, cfg: dict, eps: float = 1e-6,
                 theta: float = 1000000.0, moe_map: dict | None = None):
        self.t = {k: np.asarray(v, dtype=np.float16) for k, v in tensors.items()}
        self.cfg = cfg
        self.n_heads = int(cfg.get("num_attention_heads", 14))
        self.n_kv = int(cfg.get("num_key_value_heads", self.n_heads))
        self.n_layer = int(cfg.get("num_hidden_layers", 24))
        self.eps, self.theta = eps, theta
        self._wcache = {}
        self.hd = self.t["model.embed_tokens.weight"].shape[1] // self.n_heads
        head = self.t.get("lm_head.weight")
        self.head = self.t["model.embed_tokens.weight"] if head is None else head
        self.moe = {}
        for lyr in range(self.n_layer):
            if f"model.layers.{lyr}.mlp.experts.gate_up_proj" in self.t:
                mm = (moe_map or {}).get(str(lyr), (moe_map or {}).get(lyr))
                if mm is None:
                    raise KeyError(f"layer {lyr} has virtual-MoE experts but no map")
                self.moe[lyr] = {"experts": int(mm["experts"]), "ie": int(mm["ie"]),
                                 "top_k": int(mm["top_k"])}

    def W(self, name):
        """fp32 transposed weight, converted once and kept (chat.py:223-230)."""
        w = self._wcache.get(name)
        if w is None:
            w = self._wcache[name] = self.t[name].T.astype(np.float32)
        return w

    def layer(self, x, lyr, cache, pos0, attn_bias=None, pos_override=None):
        t, hd, nh, nk, W = self.t, self.hd, self.n_heads, self.n_kv, self.W
        p = f"model.layers.{lyr}."
        h = rmsnorm(x, t[p + "input_layernorm.weight"], self.eps)
        q = h @ W(p + "self_attn.q_proj.weight")
        k = h @ W(p + "self_attn.k_proj.weight")
        v = h @ W(p + "self_attn.v_proj.weight")
        sq = q.shape[0]
        q = q.reshape(sq, nh, hd)
        k = k.reshape(k.shape[0], nk, hd)
        v = v.reshape(v.shape[0], nk, hd)
        row_pos = (np.asarray(pos_override).reshape(-1) if pos_override is not None
                   else pos0 + np.arange(sq))
        ang = (rope_angles_at(hd, row_pos, self.theta) if pos_override is not None
               else rope_freqs(hd, sq, self.theta, pos0))
        q = apply_rope(q, ang[:, None, :])
        k = apply_rope(k, ang[:, None, :])
        rep = nh // nk
        k = np.repeat(k, rep, axis=1)
        v = np.repeat(v, rep, axis=1)
        if lyr in cache:
            k = np.concatenate([cache[lyr][0], k], axis=0)
            v = np.concatenate([cache[lyr][1], v], axis=0)
        cache[lyr] = (k, v)
        n_prev = k.shape[0] - sq
        key_pos = np.concatenate([np.arange(n_prev), row_pos]) if n_prev > 0 else row_pos
        allow = key_pos[None, :] <= row_pos[:, None]
        bias = np.where(allow, 0.0, -np.inf).astype(np.float32)
        if attn_bias is not None:
            bias = np.minimum(bias, attn_bias.astype(np.float32))
        qh = q.transpose(1, 0, 2)
        kh = k.transpose(1, 2, 0)
        vh = v.transpose(1, 0, 2)
        sc = qh @ kh / max(hd ** 0.5, 1e-6)
        e = np.exp(sc + bias[None] - (sc + bias[None]).max(-1, keepdims=True))
        a = e / e.sum(-1, keepdims=True)
        o = (a @ vh).transpose(1, 0, 2).reshape(sq, nh * hd)
        o = o @ W(p + "self_attn.o_proj.weight")
        x = x + o.astype(np.float32)
        h = rmsnorm(x, t[p + "post_attention_layernorm.weight"], self.eps)
        if lyr in self.moe:
            mc = self.moe[lyr]
            E, Ie = mc["experts"], mc["ie"]
            mp = p + "mlp."
            gu = np.asarray(t[mp + "experts.gate_up_proj"], dtype=np.float32).reshape(E, 2 * Ie, -1)
            dn = np.asarray(t[mp + "experts.down_proj"], dtype=np.float32).reshape(E, Ie, -1)
            rw = np.asarray(t[mp + "gate.weight"], dtype=np.float32)
            rb = (np.asarray(t[mp + "gate_bias"], dtype=np.float32)
                  if mp + "gate_bias" in t else None)
            d, _ = moe_grouped_forward(h.astype(np.float32), gu, dn, rw, mc["top_k"],
                                       router_b=rb, router_feat=mc.get("router_feat", "raw"))
            return x + d
        g = h @ W(p + "mlp.gate_proj.weight")
        u = h @ W(p + "mlp.up_proj.weight")
        d = (g / (1.0 + np.exp(-np.clip(g, -40, 40)))) * u
        d = d @ W(p + "mlp.down_proj.weight")
        return x + d

    # -- greedy drivers ------------------------------------------------------
    def embed(self):
        return self.t["model.embed_tokens.weight"].astype(np.float32)

    def head_t(self):
        return self.head.T.astype(np.float32)


def generate(model: OracleModel, ids: list[int], max_tokens: int,
             stop_ids=(151643,), return_logits: bool = False):
    """Greedy ``generate`` (chat.py:307-407; pick at temperature 0 = argmax of
    float64 logits, :330-339). Returns tokens (and per-step logits)."""
    emb, head_t = model.embed(), model.head_t()
    cache: dict = {}
    h = emb[np.array(ids)]
    for lyr in range(model.n_layer):
        h = model.layer(h, lyr, cache, 0)
    pos, out, logits = len(ids), [], []
    buf = np.empty((1, head_t.shape[1]), dtype=np.float32)
    while len(out) < max_tokens:
        np.dot(h[-1:], head_t, out=buf)
        lg = buf[0].copy()
        if return_logits:
            logits.append(lg)
        nxt = int(np.argmax(np.asarray(lg, dtype=np.float64)))
        if nxt in stop_ids:
            break
        out.append(nxt)
        h = emb[[nxt]]
        for lyr in range(model.n_layer):
            h = model.layer(h, lyr, cache, pos)
        pos += 1
    return (out, logits, cache) if return_logits else out


def common_prefix(a, b):
    """chat.py:410-415."""
    n = min(len(a), len(b))
    i = 0
    while i < n and a[i] == b[i]:
        i += 1
    return i


def generate_cached(model: OracleModel, ids: list[int], max_tokens: int,
                    state: dict | None = None, stop_ids=(151643,)):
    """Greedy ``generate_cached`` (chat.py:418-551): longest-common-prefix
    reuse, truncate on divergence, truncated replay when fully cached."""
    emb, head = model.embed(), model.head_t()
    st = state if state is not None else {"ids": [], "kv": {}, "pos": 0}
    common = common_prefix(st["ids"], ids)
    if common < len(st["ids"]):
        for lyr, (k, v) in list(st["kv"].items()):
            st["kv"][lyr] = (k[:common], v[:common])
        st["ids"] = st["ids"][:common]
        st["pos"] = common
    reused = len(st["ids"])
    delta = ids[len(st["ids"]):]
    h = emb[np.array(delta)] if len(delta) else emb[np.array(ids[-1:])]
    pos = st["pos"]
    if len(delta):
        for lyr in range(model.n_layer):
            h = model.layer(h, lyr, st["kv"], pos)
        pos += len(delta)
    else:
        pos0r = max(pos - 1, 0)
        kv_replay = {}
        for lyr, (k, v) in st["kv"].items():
            kv_replay[lyr] = (k[:pos0r], v[:pos0r]) if pos0r else (
                np.zeros((0,) + k.shape[1:], k.dtype), np.zeros((0,) + v.shape[1:], v.dtype))
        h = emb[[ids[-1]]]
        for lyr in range(model.n_layer):
            h = model.layer(h, lyr, kv_replay, pos0r)
    out = []
    buf = np.empty((1, head.shape[1]), dtype=np.float32)
    while len(out) < max_tokens:
        np.dot(h[-1:], head, out=buf)
        nxt = int(np.argmax(np.asarray(buf[0], dtype=np.float64)))
        if nxt in stop_ids:
            break
        out.append(nxt)
        h = emb[[nxt]]
        for lyr in range(model.n_layer):
            h = model.layer(h, lyr, st["kv"], pos)
        pos += 1
    st["ids"] = list(ids) + out
    st["pos"] = pos
    return out, {"prefill_reused": reused, "prefill_computed": len(delta)}, st


def pld_draft(ids: list[int], n: int = 4, gram: int = 3) -> list[int]:
    """Prompt-lookup draft (chat.py:553-569)."""
    if len(ids) < gram + 1:
        return []
    key = ids[-gram:]
    for i in range(len(ids) - gram - 1, -1, -1):
        if ids[i:i + gram] == key:
            cont = ids[i + gram:i + gram + n]
            if cont:
                return cont
    return []


def generate_spec(model: OracleModel, ids: list[int], max_tokens: int,
                  draft_n: int = 4, stop_ids=(151643,)):
    """Greedy ``generate_spec`` (chat.py:572-648): prompt-lookup drafts,
    one multi-row verify, acceptance by argmax, rollback of the KV to the
    accepted prefix (:636-638) and a single-row forward of the bonus token.
    Returns (tokens, [drafted, accepted, target_forwards, tokens_out])."""
    emb, head = model.embed(), model.head_t()
    cache: dict = {}
    h = emb[np.array(ids)]
    for lyr in range(model.n_layer):
        h = model.layer(h, lyr, cache, 0)
    pos, out = len(ids), []
    drafted_n = accepted_n = forwards = tokens_out = 0
    while len(out) < max_tokens:
        drafted = pld_draft(ids + out, draft_n)
        if not drafted:
            nxt = int(np.argmax((h[-1:] @ head)[0]))
            if nxt in stop_ids:
                break
            out.append(nxt)
            h = emb[[nxt]]
            for lyr in range(model.n_layer):
                h = model.layer(h, lyr, cache, pos)
            pos += 1
            forwards += 1
            tokens_out += 1
            continue
        drafted_n += len(drafted)
        hh = emb[np.array(drafted)]
        for lyr in range(model.n_layer):
            hh = model.layer(hh, lyr, cache, pos)
        forwards += 1
        t_lg = hh @ head
        h_lg = (h[-1:] @ head)[0]
        acc = []
        bonus = int(np.argmax(t_lg[-1]))
        for k, tok in enumerate(drafted):
            pred = h_lg if k == 0 else t_lg[k - 1]
            if int(np.argmax(pred)) == tok:
                acc.append(tok)
            else:
                bonus = int(np.argmax(pred))
                break
        accepted_n += len(acc)
        tokens_out += len(acc) + 1
        for a in acc + [bonus]:
            out.append(a)
            if a in stop_ids:
                return out, [drafted_n, accepted_n, forwards, tokens_out]
        for lyr in range(model.n_layer):
            k, v = cache[lyr]
            cache[lyr] = (k[:pos + len(acc)], v[:pos + len(acc)])
        h = emb[[bonus]]
        for lyr in range(model.n_layer):
            h = model.layer(h, lyr, cache, pos + len(acc))
        forwards += 1
        pos += len(acc) + 1
    return out[:max_tokens], [drafted_n, accepted_n, forwards, tokens_out]


def build_tree_mask(parents):
    """spec.py:56-83: 0 where a node may attend (itself, its ancestors)."""
    n = len(parents)
    mask = np.full((n, n), -np.inf, dtype=np.float32)
    for i in range(n):
        mask[i, i] = 0.0
        c = parents[i]
        while c >= 0:
            mask[i, c] = 0.0
            if parents[c] == c:
                break
            c = parents[c]
    return mask


def tree_bias(parents, depths, Lp):
    """The (N, Lp+N) additive bias verify_tree builds (eagle.py:271-282):
    every child sees the prefix (the root lives there), itself and its
    non-root ancestors among the children."""
    order = [i for i in range(len(parents)) if depths[i] >= 1]
    N = len(order)
    tm = build_tree_mask(parents)
    bias = np.full((N, Lp + N), -np.inf, dtype=np.float32)
    bias[:, :Lp] = 0.0
    gidx = {old: new for new, old in enumerate(order)}
    for ni, oi in enumerate(order):
        for oj in range(len(parents)):
            if tm[oi, oj] == 0.0 and oj != 0 and oj in gidx:
                bias[ni, Lp + gidx[oj]] = 0.0
    return order, bias


def verify_tree(model: OracleModel, cache: dict, pos: int, tree_ids, parents, depths):
    """eagle.py:259-291: one forward over the children with the ancestry bias
    and true positions; returns (logits, tree cache, hidden)."""
    emb = model.embed()
    order, bias = tree_bias(parents, depths, pos)
    x = np.stack([emb[tree_ids[i]] for i in order])
    pos_ov = np.array([pos - 1 + depths[i] for i in order])
    tc = dict(cache)
    h = x
    for lyr in range(model.n_layer):
        h = model.layer(h, lyr, tc, pos, attn_bias=bias, pos_override=pos_ov)
    return h @ model.head_t(), tc, h


def commit_rows(cache: dict, tc: dict, path_rows: list[int]):
    """The KV row gather of commit_verified (eagle.py:340-350): append the
    tree-cache rows ``Lp + gidx[node]`` of the accepted path, in path order."""
    for lyr in list(cache.keys()):
        ok, ov = cache[lyr]
        tk, tv = tc[lyr]
        Lp = ok.shape[0]
        rk = [tk[[Lp + r]] for r in path_rows]
        rv = [tv[[Lp + r]] for r in path_rows]
        cache[lyr] = (np.concatenate([ok] + rk) if rk else ok,
                      np.concatenate([ov] + rv) if rv else ov)
