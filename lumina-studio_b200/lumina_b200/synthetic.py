"""Seeded synthetic workloads for the Lumina decode path.

There is no dataset or checkpoint on this path: the workloads are seeded
random Llama-style decoders, quantized to Lumina codes. Shapes:

  * ``TINY``  — 4 layers, d 256, 4 heads x 64, SwiGLU 688, vocab 4096,
    RoPE theta 1e4 (the reference's CPU-runnable mini_lm shape).
  * ``LLAMA7B`` — 32 layers, d 4096, 32 heads x 128, SwiGLU 11008,
    vocab 32000, RoPE theta 1e4.

Weights of every 2-D matrix are N(0, 0.02) drawn in the fixed order of
``tensor_order``; RMSNorm weights are ones. Tensor names follow the HF Llama
layout that the reference's ChatModel reads (chat.py:240-303).
"""
from __future__ import annotations

import numpy as np

TINY = {"name": "tiny", "num_hidden_layers": 4, "hidden_size": 256,
        "num_attention_heads": 4, "num_key_value_heads": 4,
        "intermediate_size": 688, "vocab_size": 4096, "rope_theta": 10000.0}

LLAMA7B = {"name": "llama7b", "num_hidden_layers": 32, "hidden_size": 4096,
           "num_attention_heads": 32, "num_key_value_heads": 32,
           "intermediate_size": 11008, "vocab_size": 32000, "rope_theta": 10000.0}

# the 7B shape cut to two layers: every kernel instantiation of the 7B decode
# (head_dim 128, fp16 KV, the 32000-row head) at a size the CPU oracle runs
LLAMA7B_2L = dict(LLAMA7B, name="llama7b_2l", num_hidden_layers=2)


def tensor_order(cfg: dict) -> list[tuple[str, tuple[int, ...]]]:
    """(name, shape) in generation order."""
    d, f, v = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    nh, nk = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    hd = d // nh
    out = [("model.embed_tokens.weight", (v, d))]
    for l in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{l}."
        out += [(p + "input_layernorm.weight", (d,)),
                (p + "self_attn.q_proj.weight", (nh * hd, d)),
                (p + "self_attn.k_proj.weight", (nk * hd, d)),
                (p + "self_attn.v_proj.weight", (nk * hd, d)),
                (p + "self_attn.o_proj.weight", (d, nh * hd)),
                (p + "post_attention_layernorm.weight", (d,)),
                (p + "mlp.gate_proj.weight", (f, d)),
                (p + "mlp.up_proj.weight", (f, d)),
                (p + "mlp.down_proj.weight", (d, f))]
    out.append(("lm_head.weight", (v, d)))
    return out


def host_weights(cfg: dict, seed: int = 0) -> dict[str, np.ndarray]:
    """fp32 weights on the host (for shapes the CPU can hold comfortably)."""
    rng = np.random.default_rng(seed)
    w = {}
    for name, shape in tensor_order(cfg):
        if len(shape) == 1:
            w[name] = np.ones(shape, dtype=np.float32)
        else:
            w[name] = (rng.standard_normal(shape) * 0.02).astype(np.float32)
    return w


def virtual_moe_weights(cfg: dict, experts: int = 8, top_k: int = 2, seed: int = 0,
                        router_std: float = 0.02) -> tuple[dict[str, np.ndarray], dict]:
    """``host_weights`` with every layer's SwiGLU MLP split into ``experts``
    routed experts, stored flat as the reference's virtual-MoE converter
    writes them (virtual_moe.py:140-147, 228-235): expert e owns the
    contiguous neurons [e*Ie, (e+1)*Ie), Ie = ffn / experts;
    ``experts.gate_up_proj`` (E*2Ie, D) holds its gate rows then its up rows,
    ``experts.down_proj`` (E*Ie, D) the transposed down columns. The router
    ``gate.weight`` (E, D) and ``gate_bias`` (E) are N(0, router_std), drawn
    after the dense weights from seed + 1000. Returns (arrays, virtual_moe
    header map keyed by tensor prefix, as write_lumina stores it)."""
    f, d = cfg["intermediate_size"], cfg["hidden_size"]
    if f % experts:
        raise ValueError(f"ffn {f} does not split into {experts} equal experts")
    ie = f // experts
    w = host_weights(cfg, seed)
    rng = np.random.default_rng(seed + 1000)
    meta = {}
    for l in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{l}.mlp."
        g = w.pop(p + "gate_proj.weight")
        u = w.pop(p + "up_proj.weight")
        dn = w.pop(p + "down_proj.weight")
        w[p + "experts.gate_up_proj"] = np.concatenate(
            [np.concatenate([g[e * ie:(e + 1) * ie], u[e * ie:(e + 1) * ie]]) for e in range(experts)])
        w[p + "experts.down_proj"] = np.ascontiguousarray(
            np.concatenate([dn[:, e * ie:(e + 1) * ie].T for e in range(experts)]))
        w[p + "gate.weight"] = (rng.standard_normal((experts, d)) * router_std).astype(np.float32)
        w[p + "gate_bias"] = (rng.standard_normal(experts) * router_std).astype(np.float32)
        meta[p] = {"experts": experts, "ie": ie, "top_k": top_k, "router_feat": "raw", "layer": str(l)}
    return w, meta


def random_int4_payloads(cfg: dict, seed: int = 0, group: int = 64) -> dict:
    """convert_arrays-style payloads ``{name: ("raw", fp32) | ("int4",
    (codes, scales))}`` of a seeded decoder whose projections are drawn
    directly as Lumina int4 records: codes uniform over 0..15 (uint8,
    (rows, cols)), group scales uniform in [0.03, 0.06) rounded to fp16
    values (stored F32, as the converter writes them), so that the weights
    s * (2c - 15) / 15 have a standard deviation near 0.02. Embedding and
    lm_head are raw N(0, 0.02); RMSNorm weights are 1 + N(0, 0.1). Drawn in
    ``tensor_order`` from one generator. Used for parity cases at full model
    width, where running the quantizer over every matrix would dominate."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in tensor_order(cfg):
        if len(shape) == 1:
            out[name] = ("raw", (1.0 + 0.1 * rng.standard_normal(shape)).astype(np.float32))
        elif "embed" in name or "lm_head" in name:
            out[name] = ("raw", (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)))
        else:
            rows, cols = shape
            codes = rng.integers(0, 16, (rows, cols), dtype=np.uint8)
            ng = -(-cols // group)
            scales = rng.uniform(0.03, 0.06, (rows, ng)).astype(np.float16).astype(np.float32)
            out[name] = ("int4", (codes, scales))
    return out


def prompt_ids(cfg: dict, n: int, seed: int = 0) -> list[int]:
    """Uniform random prompt ids from a seeded generator."""
    rng = np.random.default_rng(seed + 1)
    return [int(t) for t in rng.integers(0, cfg["vocab_size"], n)]


def hf_cfg(cfg: dict) -> dict:
    """The HF-style config dict the reference's ChatModel reads."""
    return {k: cfg[k] for k in ("num_hidden_layers", "hidden_size", "num_attention_heads",
                                "num_key_value_heads", "vocab_size", "intermediate_size")}


# ---------------------------------------------------------------------------
# Full-size quantized workloads, generated on the GPU
# ---------------------------------------------------------------------------
_MULTIPLIERS = (1.0, 0.8, 0.65, 0.5, 0.4, 0.3, 0.2)  # ptq_ladder.py:235


def _nearest_level(wn, lv, L: int):
    """Index of the level nearest to each of `wn`, the first index winning a
    tie: ``np.abs(wn[..., None] - lv).argmin(-1)`` of ptq_ladder.py:238-239,
    314, without the (..., L + 1) distance tensor. The nearest level is one
    of the three around ``floor((wn + 1) L / 2)`` (the floor can be off by
    one where wn sits on a level); they are compared in index order."""
    import torch
    k = torch.clamp(torch.floor((wn + 1.0) * (L / 2.0)), 0, L).long()
    best = torch.clamp(k - 1, 0, L)
    best_d = (wn - lv[best]).abs()
    for cand in (k, torch.clamp(k + 1, 0, L)):
        d = (wn - lv[cand]).abs()
        take = d < best_d
        best = torch.where(take, cand, best)
        best_d = torch.where(take, d, best_d)
    return best


def _quantize_gpu(w, bits: int, group: int):
    """Lumina codes and scales of one weight, the reference's RTN + MSE scale
    search (ptq_ladder.py:215-249, 370-399 with H = I; seven absmax
    multipliers, the first minimum wins) in fp64 on the weight's device:
    codes are the nearest levels of w / s with the unrounded scale, and the
    stored scale is s rounded to fp32 and then to fp16, as the file writer
    does. `w` is a (rows, cols) float32 tensor; a last group narrower than
    `group` is scored over its own columns. Returns (codes uint8 (rows,
    cols), scales float32 (rows, ceil(cols/group))). This makes benchmark
    inputs: it is the reference's quantizer restated in torch, not code
    under test."""
    import torch
    L = (1 << bits) - 1
    # the reference's levels, np.linspace(-1, 1, 2^b) (ptq_ladder.py:58-59)
    lv = torch.from_numpy(np.linspace(-1.0, 1.0, L + 1)).to(w.device)
    rows, cols = w.shape
    ng = -(-cols // group)
    pad = ng * group - cols
    w = w.double()
    if pad:
        w = torch.nn.functional.pad(w, (0, pad))  # zeros never raise a group's absmax
    wg = w.view(rows, ng, group)
    valid = torch.ones(ng, group, device=w.device, dtype=torch.bool)
    if pad:
        valid[-1, group - pad:] = False
    cnt = valid.sum(-1).double()
    amax = wg.abs().amax(-1).clamp_min(1e-12)
    best_e = best_s = None
    for f in _MULTIPLIERS:
        s = (amax * f).clamp_min(1e-12)
        wn = wg / s[..., None]
        err = torch.where(valid, (wn - lv[_nearest_level(wn, lv, L)]) ** 2, 0.0)
        e = err.sum(-1) / cnt
        del wn, err
        if best_e is None:
            best_e, best_s = e, s
        else:
            take = e < best_e
            best_e = torch.where(take, e, best_e)
            best_s = torch.where(take, s, best_s)
    c = _nearest_level(wg / best_s[..., None], lv, L).to(torch.uint8)
    s16 = best_s.float().half().float()
    return c.view(rows, ng * group)[:, :cols].contiguous(), s16


def _pack_gpu(c, bits: int):
    """Codes (rows, cols) uint8 -> the file's packed bytes: int4 nibbles with
    the even column in the low nibble (adapters/lumina.py:20-27), int2 four
    per byte from bit 0 (adapters/lumina.py:30-40), int3 one byte per code."""
    if bits == 4:
        return c[:, 0::2] | (c[:, 1::2] << 4)
    if bits == 2:
        return c[:, 0::4] | (c[:, 1::4] << 2) | (c[:, 2::4] << 4) | (c[:, 3::4] << 6)
    if bits == 3:
        return c
    raise ValueError(f"bits {bits}")


class QuantizedRecords:
    """Lazily generated records of a seeded random decoder (every 2-D matrix
    N(0, 0.02), projections Lumina-quantized with fp16-valued group scales,
    embedding and lm_head raw fp32, RMSNorm weights ones), as the mapping
    ``CudaChatModel._from_records`` reads. Each tensor is drawn on the GPU
    from its own seed (seed, index in ``tensor_order``) when first asked for
    and is not kept, so a 7B model never sits on the host as a whole."""

    def __init__(self, cfg: dict, bits: int = 4, group: int = 64, seed: int = 0, device: int = 0,
                 moe: tuple[int, int] | None = None):
        """``moe = (experts, top_k)`` makes every layer a virtual-MoE layer:
        the MLP's gate/up/down become ``experts.gate_up_proj`` (E*2Ie, D)
        and ``experts.down_proj`` (E*Ie, D), quantized like the other
        projections, plus a raw router ``gate.weight`` (E, D) and
        ``gate_bias`` (E), all N(0, 0.02); ``moe_map`` then holds the
        per-layer (experts, ie, top_k)."""
        self.cfg, self.bits, self.group, self.seed, self.device = cfg, bits, group, seed, device
        order = tensor_order(cfg)
        self.moe_map = {}
        if moe:
            e, k = moe
            f, d = cfg["intermediate_size"], cfg["hidden_size"]
            if f % e:
                raise ValueError(f"ffn {f} does not split into {e} equal experts")
            ie = f // e
            out = []
            for name, shape in order:
                if ".mlp.gate_proj." in name:
                    p = name[: -len("gate_proj.weight")]
                    out += [(p + "experts.gate_up_proj", (e * 2 * ie, d)), (p + "experts.down_proj", (e * ie, d)),
                            (p + "gate.weight", (e, d)), (p + "gate_bias", (e,))]
                    self.moe_map[int(name.split(".")[2])] = {"experts": e, "ie": ie, "top_k": k}
                elif ".mlp.up_proj." not in name and ".mlp.down_proj." not in name:
                    out.append((name, shape))
            order = out
        self.order = {n: (i, s) for i, (n, s) in enumerate(order)}

    def __contains__(self, name):
        return name in self.order

    def get(self, name, default=None):
        return self[name] if name in self.order else default

    def __getitem__(self, name):
        import torch
        from .loader import Record
        idx, shape = self.order[name]
        if len(shape) == 1 and not name.endswith("gate_bias"):
            return Record(name, "raw", shape, data=np.ones(shape, np.float32))
        g = torch.Generator(device=f"cuda:{self.device}")
        g.manual_seed(self.seed * 100003 + idx)
        w = torch.randn(shape, generator=g, device=f"cuda:{self.device}", dtype=torch.float32) * 0.02
        if "embed" in name or "lm_head" in name or name.endswith((".gate.weight", "gate_bias")):
            return Record(name, "raw", shape, data=w.cpu().numpy())
        c, s = _quantize_gpu(w, self.bits, self.group)
        packed = _pack_gpu(c, self.bits).contiguous().cpu().numpy().reshape(-1)
        pack = {4: "nibble", 2: "2bit", 3: "none"}[self.bits]
        return Record(name, f"int{self.bits}", shape, group=self.group, pack=pack, codes=packed,
                      scales=s.cpu().numpy())
