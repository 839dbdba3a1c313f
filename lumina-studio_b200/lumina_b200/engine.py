"""CudaChatModel: the reference ChatModel's decode path on liblumina_cuda.

Mirrors the interface of src/lumina_framework/chat.py for this path:

  * ``CudaChatModel.from_lumina(path, cfg, tok, ..., theta=...)`` — builds
    straight from a `.lumina` file (codes go to the device packed); the
    ``n_heads`` / ``n_kv`` arguments are fallbacks behind the config
    (chat.py:184-188); ``theta`` defaults to 1e6 as the reference does
    (chat.py:119,131) and must be passed for other models.
  * ``_layer(x, lyr, cache, pos0, attn_bias=None, pos_override=None)`` — the
    per-layer drop-in (chat.py:232-304); ``cache`` is the model's
    ``DeviceKV``, whose ``cache[lyr] = (k, v)`` entries expose ``.shape``,
    ``[:n]`` and ``np.asarray`` like the reference's numpy tuples.
  * ``generate`` / ``generate_cached`` / ``generate_spec`` / ``verify_tree``
    / ``commit_verified`` — replacements of the reference drivers
    (chat.py:307-648, eagle.py:259-357) with the KV slicing and row gathers
    done as block-table operations on the device; the sampler ``pick`` stays
    on the host. The reference's own drivers build a numpy ``cache`` dict
    and cannot run on this model, so these are the drivers to call.

There is no CPU path: without the CUDA library these raise ``LuminaError``.
"""
from __future__ import annotations

import ctypes
import re
import time

import numpy as np

from . import cuda
from .cuda import LuminaError, ModelConfig, check, ptr
from .loader import LuminaFile, upload_record


def rope_tables(head_dim: int, n_pos: int, theta: float):
    """cos / sin tables with the reference's float32 arithmetic
    (chat.py:69-85): freq_i = 1 / theta ** (float32(2i) / hd), angle =
    float32(p) * freq_i, numpy float32 cos / sin."""
    freqs = 1.0 / (theta ** (np.arange(0, 2 * (head_dim // 2), 2).astype(np.float32) / head_dim))
    ang = np.outer(np.arange(n_pos, dtype=np.float32), freqs)
    return np.ascontiguousarray(np.cos(ang), np.float32), np.ascontiguousarray(np.sin(ang), np.float32)


class _KVView:
    """k or v rows [0, n) of one layer, as the reference's (T, H, hd) array."""

    def __init__(self, kv, lyr, which, n):
        self.kv, self.lyr, self.which, self.n = kv, lyr, which, n

    @property
    def shape(self):
        m = self.kv.model
        return (self.n, m.n_heads_local, m.hd)

    @property
    def dtype(self):
        return np.dtype(np.float32)

    def __len__(self):
        return self.n

    def __getitem__(self, key):
        if isinstance(key, slice) and key.step in (None, 1) and (key.start in (None, 0)):
            stop = self.n if key.stop is None else max(0, min(self.n, key.stop if key.stop >= 0 else self.n + key.stop))
            return _KVView(self.kv, self.lyr, self.which, stop)
        return np.asarray(self)[key]

    def __array__(self, dtype=None, copy=None):
        k, v = self.kv.read(self.lyr, 0, self.n)
        a = k if self.which == 0 else v
        return a.astype(dtype) if dtype is not None else a


class DeviceKV:
    """Per-layer KV cache on the device with the chat.py dict contract.

    ``kv[lyr]`` is a (k, v) pair of views; assigning views with fewer rows
    truncates (chat.py:442-445, 636-638). Every layer shares one block table,
    so a truncation applies to the whole model once every layer has been
    assigned the same length (the reference loops over all layers).
    """

    def __init__(self, model):
        self.model = model
        self._pending: dict[int, int] = {}

    def _len(self, lyr=None):
        return self.model.kv_length(lyr)

    def __contains__(self, lyr):
        return 0 <= lyr < self.model.n_layer and self._len(lyr) > 0

    def __getitem__(self, lyr):
        n = self._len(lyr)
        return (_KVView(self, lyr, 0, n), _KVView(self, lyr, 1, n))

    def __setitem__(self, lyr, kv):
        n = len(kv[0])
        if n > self._len(lyr):
            raise ValueError("DeviceKV only shrinks by assignment (rows are appended by _layer)")
        self._pending[lyr] = n
        if len(self._pending) == self.model.n_layer:
            lens = set(self._pending.values())
            self._pending.clear()
            if len(lens) != 1:
                raise ValueError("layers truncated to different lengths")
            self.model.kv_truncate(lens.pop())

    def keys(self):
        return [l for l in range(self.model.n_layer) if l in self]

    def items(self):
        return [(l, self[l]) for l in self.keys()]

    def __iter__(self):
        return iter(self.keys())

    def __len__(self):
        return len(self.keys())

    def read(self, lyr, start, n):
        return self.model.kv_read(lyr, start, n)


def gather_peer_handles(handle: bytes, group=None) -> list:
    """Every rank's 64-byte exchange-region handle, in rank order, over the
    torch.distributed group. A rank that never joins (or died) makes this
    raise -- a connection error, or the group's timeout -- instead of waiting
    forever; create the group with a short timeout."""
    import torch.distributed as dist
    if not isinstance(handle, (bytes, bytearray)) or len(handle) != 64:
        raise LuminaError(1, "peer handle must be 64 bytes")
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(handle), group=group)
    for r, h in enumerate(out):
        if not isinstance(h, (bytes, bytearray)) or len(h) != 64:
            raise LuminaError(5, "peer handle exchange: rank %d sent %r" % (r, type(h).__name__))
    return [bytes(h) for h in out]


def moe_map_from_header(header: dict) -> dict:
    """{layer: entry} from a .lumina header's "virtual_moe" map, whose keys
    are tensor-name prefixes (serve.py:1357-1366)."""
    out = {}
    for pfx, mm in (header.get("virtual_moe") or {}).items():
        mt = re.search(r"layers\.(\d+)\.", str(pfx))
        if mt:
            out[int(mt.group(1))] = mm
    return out


def moe_layers(recs: dict, n_layer: int, moe_map: dict | None) -> dict:
    """Layers holding virtual-MoE experts -> (experts, ie, top_k), with the
    reference's rule (chat.py:157-183): an experts tensor without a map
    entry for its layer is an error."""
    out = {}
    for l in range(n_layer):
        if f"model.layers.{l}.mlp.experts.gate_up_proj" not in recs:
            continue
        mm = (moe_map or {}).get(l, (moe_map or {}).get(str(l)))
        if mm is None:
            raise KeyError(f"layer {l} has virtual-MoE experts but no virtual_moe header entry (experts/ie/top_k)")
        out[l] = {"experts": int(mm["experts"]), "ie": int(mm["ie"]), "top_k": int(mm["top_k"])}
    return out


class CudaChatModel:
    """The reference ChatModel (chat.py:106-304) with its decode path on a B200."""

    def __init__(self):
        raise TypeError("use CudaChatModel.from_lumina / from_payloads")

    # -- construction -----------------------------------------------------
    @classmethod
    def _shell(cls, cfg, tok, n_heads, n_kv, eps, theta, device, kv_fp16, max_seq, max_rows,
               block_size, tp_rank, tp_size, d_model, ffn, vocab):
        lib = cuda.ensure_device(device)
        obj = cls.__new__(cls)
        obj.lib, obj.device, obj.cfg, obj.tok = lib, device, cfg, tok
        obj.n_heads = int(cfg.get("num_attention_heads", n_heads))
        obj.n_kv = int(cfg.get("num_key_value_heads", obj.n_heads))
        obj.n_layer = int(cfg.get("num_hidden_layers", 24))
        obj.eps, obj.theta = eps, theta
        obj.d = int(d_model)
        obj.hd = obj.d // obj.n_heads
        obj.vocab = int(vocab)
        obj.tp_rank, obj.tp_size = tp_rank, tp_size
        obj.n_heads_local = obj.n_heads // tp_size
        obj.max_seq, obj.max_rows = max_seq, max_rows
        c = ModelConfig(n_layer=obj.n_layer, d_model=obj.d, n_heads=obj.n_heads, n_kv=obj.n_kv,
                        head_dim=obj.hd, ffn=int(ffn), vocab=obj.vocab, eps=eps, theta=theta,
                        kv_fp16=1 if kv_fp16 else 0, block_size=block_size, max_seq=max_seq,
                        max_rows=max_rows, tp_rank=tp_rank, tp_size=tp_size)
        h = ctypes.c_void_p()
        check(lib.lumina_model_create(device, ctypes.byref(c), ctypes.byref(h)), lib)
        obj.h = h
        obj.kv = DeviceKV(obj)
        obj._logits = np.empty(obj.vocab, dtype=np.float32)
        obj._embed = None
        obj._finalized = False
        return obj

    def _set_tensor(self, name, arr):
        a = np.ascontiguousarray(arr, dtype=np.float32)
        rows, cols = (a.shape[0], int(np.prod(a.shape[1:]))) if a.ndim > 1 else (1, a.shape[0])
        check(self.lib.lumina_model_set_tensor(self.h, name.encode(), ptr(a, ctypes.c_float), rows, cols),
              self.lib)

    def _set_weight(self, name, w):
        check(self.lib.lumina_model_set_weight(self.h, name.encode(), w.handle), self.lib)
        w.release()

    def _finalize(self, embed):
        cos, sin = rope_tables(self.hd, self.max_seq + 1, self.theta)
        self._set_tensor("rope.cos", cos)
        self._set_tensor("rope.sin", sin)
        check(self.lib.lumina_model_finalize(self.h), self.lib)
        # host copy of the fp16-rounded embedding for drop-in callers that
        # index model.t["model.embed_tokens.weight"] (chat.py:321)
        self._embed = np.asarray(embed, dtype=np.float16)
        self.t = {"model.embed_tokens.weight": self._embed}
        self._finalized = True

    @classmethod
    def from_lumina(cls, path: str, cfg: dict, tok=None, n_heads: int = 14, n_kv: int = 2,
                    eps: float = 1e-6, theta: float = 1000000.0, device: int = 0,
                    kv_fp16: bool = False, max_seq: int = 4096, max_rows: int = 128,
                    block_size: int = 16, tp_rank: int = 0, tp_size: int = 1, moe_map: dict | None = None):
        """``moe_map`` {layer: {"experts", "ie", "top_k"}} defaults to the
        file header's "virtual_moe" entries, keyed by layer as
        serve._api_load_lumina builds it (serve.py:1357-1366)."""
        with LuminaFile(path) as f:
            recs = {n: f.record(n) for n in f.names()}
            if moe_map is None:
                moe_map = moe_map_from_header(f.header)
            shard = f.header.get("tp_shard")
            if shard is not None and (int(shard["rank"]), int(shard["size"])) != (tp_rank, tp_size):
                raise LuminaError(1, "%s holds the shard of rank %s of %s, not %d of %d"
                                  % (path, shard["rank"], shard["size"], tp_rank, tp_size))
            return cls._from_records(recs, cfg, tok, n_heads, n_kv, eps, theta, device, kv_fp16,
                                     max_seq, max_rows, block_size, tp_rank, tp_size, moe_map=moe_map,
                                     presharded=shard is not None)

    @classmethod
    def from_payloads(cls, payloads: dict, cfg: dict, tok=None, group_size: int = 64, **kw):
        """Build from convert_arrays-style payloads ``{name: ("raw", fp32) |
        (kind, (codes, scales))}`` without writing a file (codes are packed
        to the file layout first)."""
        from .loader import Record
        from . import packing
        recs = {}
        for name, (kind, payload) in payloads.items():
            if kind == "raw":
                a = np.asarray(payload, dtype=np.float32)
                recs[name] = Record(name, "raw", a.shape, data=a)
            else:
                codes, scales = payload
                blob, pack, shape = packing.to_file_layout(kind, codes)
                recs[name] = Record(name, kind, shape, group=group_size, pack=pack, codes=blob,
                                    scales=np.asarray(scales, np.float32))
        return cls._from_records(recs, cfg, tok, kw.pop("n_heads", 14), kw.pop("n_kv", 2),
                                 kw.pop("eps", 1e-6), kw.pop("theta", 1000000.0), kw.pop("device", 0),
                                 kw.pop("kv_fp16", False), kw.pop("max_seq", 4096),
                                 kw.pop("max_rows", 128), kw.pop("block_size", 16),
                                 kw.pop("tp_rank", 0), kw.pop("tp_size", 1), moe_map=kw.pop("moe_map", None))

    @classmethod
    def _from_records(cls, recs, cfg, tok, n_heads, n_kv, eps, theta, device, kv_fp16, max_seq,
                      max_rows, block_size, tp_rank, tp_size, moe_map=None, presharded=False):
        """``presharded``: the records already are this rank's shard (a file
        written by shards.write_tp_shards), so they are not sliced again."""
        from . import sharding
        emb = recs["model.embed_tokens.weight"]
        if emb.kind != "raw":
            raise LuminaError(3, "quantized embeddings are not on this path (lumina_convert keeps them raw)")
        d_model = emb.shape[1]
        nl = int(cfg.get("num_hidden_layers", 24))
        moe = moe_layers(recs, nl, moe_map)
        dense = [l for l in range(nl) if l not in moe]
        ffn = (recs[f"model.layers.{dense[0]}.mlp.gate_proj.weight"].shape[0] if dense
               else max(m["ie"] for m in moe.values()))
        head = recs.get("lm_head.weight")
        vocab = (head or emb).shape[0] * (tp_size if presharded and head is not None else 1)
        obj = cls._shell(cfg, tok, n_heads, n_kv, eps, theta, device, kv_fp16, max_seq, max_rows,
                         block_size, tp_rank, tp_size, d_model, ffn, vocab)
        obj.moe = moe
        try:
            obj._set_tensor("model.embed_tokens.weight", emb.data)
            if head is not None:
                if head.kind != "raw":
                    raise LuminaError(3, "quantized lm_head is not on this path")
                obj._set_tensor("lm_head.weight", head.data if presharded
                                else sharding.vocab_shard(head.data, tp_rank, tp_size))
            for l in range(nl):
                p = f"model.layers.{l}."
                for nm in ("input_layernorm.weight", "post_attention_layernorm.weight"):
                    obj._set_tensor(p + nm, recs[p + nm].data)
                mlp = ("mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight")
                if l in moe:
                    mc = moe[l]
                    check(obj.lib.lumina_model_set_moe(obj.h, l, mc["experts"], mc["ie"], mc["top_k"]), obj.lib)
                    obj._set_tensor(p + "mlp.gate.weight", recs[p + "mlp.gate.weight"].data)
                    if p + "mlp.gate_bias" in recs:
                        obj._set_tensor(p + "mlp.gate_bias", recs[p + "mlp.gate_bias"].data)
                    for nm in ("mlp.experts.gate_up_proj", "mlp.experts.down_proj"):
                        rec = recs[p + nm]
                        if rec.kind == "raw":
                            raise LuminaError(3, f"{p + nm} is stored raw; only packed experts are built")
                        if not presharded:  # expert parallelism: this rank's experts
                            rec = sharding.expert_shard(rec, mc["experts"], tp_rank, tp_size)
                        obj._set_weight(p + nm, upload_record(rec, device))
                    mlp = ()
                for nm in ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                           "self_attn.o_proj.weight") + mlp:
                    rec = recs[p + nm]
                    if rec.kind == "raw":
                        raise LuminaError(3, f"{p + nm} is stored raw; only packed projections are built")
                    if not presharded:
                        rec = sharding.shard_record(rec, nm, tp_rank, tp_size, obj.hd)
                    obj._set_weight(p + nm, upload_record(rec, device))
            obj._finalize(emb.data)
        except Exception:
            obj.close()
            raise
        return obj

    def init_tp(self, group=None):
        """Join the other ranks of this tensor-parallel model: every rank's
        exchange-region handle goes to every rank over the torch.distributed
        group (rank r of the group must hold shard tp_rank = r), and each
        rank maps its peers' regions; the sums after o_proj / down_proj and
        the logits gather then run over peer memory. No-op when the model is
        not sharded."""
        if self.tp_size <= 1:
            return
        h = (ctypes.c_uint8 * 64)()
        check(self.lib.lumina_model_peer_handle(self.h, h), self.lib)
        allh = b"".join(gather_peer_handles(bytes(h), group))
        buf = (ctypes.c_uint8 * len(allh)).from_buffer_copy(allh)
        check(self.lib.lumina_model_init_peers(self.h, buf), self.lib)

    def close(self):
        if getattr(self, "h", None):
            self.lib.lumina_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    # -- KV ------------------------------------------------------------------
    def kv_length(self, lyr=None) -> int:
        n = ctypes.c_int()
        check(self.lib.lumina_kv_length(self.h, -1 if lyr is None else int(lyr), ctypes.byref(n)), self.lib)
        return n.value

    def kv_truncate(self, n: int):
        check(self.lib.lumina_kv_truncate(self.h, int(n)), self.lib)

    def kv_read(self, lyr, start, n):
        k = np.empty((n, self.n_heads_local, self.hd), np.float32)
        v = np.empty_like(k)
        check(self.lib.lumina_kv_read(self.h, int(lyr), int(start), int(n), ptr(k, ctypes.c_float),
                                      ptr(v, ctypes.c_float)), self.lib)
        return k, v

    def kv_commit_rows(self, base, src):
        s = np.ascontiguousarray(src, dtype=np.int32)
        check(self.lib.lumina_kv_commit_rows(self.h, int(base), ptr(s, ctypes.c_int), len(s)), self.lib)

    def kv_attend(self, lyr, q):
        """Single-query attention of q (n_heads_local, hd) over every cached row
        of layer ``lyr`` (chat.py:264-281 with one row, no bias), on the
        device's decode-attention kernel."""
        q = np.ascontiguousarray(q, dtype=np.float32).reshape(self.n_heads_local, self.hd)
        out = np.empty_like(q)
        check(self.lib.lumina_kv_attend(self.h, int(lyr), ptr(q, ctypes.c_float), ptr(out, ctypes.c_float)),
              self.lib)
        return out

    # -- forwards ------------------------------------------------------------
    def _layer(self, x, lyr, cache, pos0, attn_bias=None, pos_override=None):
        """chat.py:232-304 on the device. ``cache`` must be this model's
        DeviceKV (or a dict built from its views, as eagle.verify_tree makes
        with ``dict(cache)``); the new K/V rows are appended on the device."""
        import torch
        x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
        n = x.shape[0]
        xd = torch.from_numpy(x).to(f"cuda:{self.device}")
        po = None
        if pos_override is not None:
            po = np.ascontiguousarray(np.asarray(pos_override).reshape(-1), dtype=np.int32)
        b = None
        if attn_bias is not None:
            b = np.ascontiguousarray(attn_bias, dtype=np.float32)
            b = np.where(np.isnan(b), np.float32(0), b)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(self.lib.lumina_layer_forward(self.h, int(lyr), xd.data_ptr(), n, int(pos0),
                                            ptr(po, ctypes.c_int) if po is not None else None,
                                            ptr(b, ctypes.c_float) if b is not None else None,
                                            stream), self.lib)
        return xd.cpu().numpy()

    def forward(self, tokens, pos0: int, all_rows: bool = False, pos_override=None,
                attn_bias=None) -> np.ndarray:
        """Embed + every layer + head logits (last row, or every row); with
        ``pos_override`` / ``attn_bias`` the tree-verification forward."""
        t = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        out = np.empty((t.size if all_rows else 1, self.vocab), np.float32)
        po = b = None
        if pos_override is not None:
            po = np.ascontiguousarray(np.asarray(pos_override).reshape(-1), dtype=np.int32)
        if attn_bias is not None:
            b = np.ascontiguousarray(attn_bias, dtype=np.float32)
        check(self.lib.lumina_forward(self.h, ptr(t, ctypes.c_int), t.size, int(pos0),
                                      ptr(po, ctypes.c_int) if po is not None else None,
                                      ptr(b, ctypes.c_float) if b is not None else None,
                                      ptr(out, ctypes.c_float), 1 if all_rows else 0), self.lib)
        return out

    def decode_step(self, token: int, want_logits: bool = True):
        """One graph-replayed greedy step at the current KV length."""
        am = ctypes.c_int()
        check(self.lib.lumina_decode_step(self.h, int(token),
                                          ptr(self._logits, ctypes.c_float) if want_logits else None,
                                          ctypes.byref(am)), self.lib)
        return (self._logits if want_logits else None), am.value

    def decode_greedy(self, token: int, n: int, timed: bool = False):
        """n greedy steps with the argmax fed back on the device: one graph
        replay per token and one host copy of the n tokens at the end. Token
        i+1 is the argmax of the logits after token i (the first one is
        `token`); the KV grows by n rows. With ``timed`` also returns the
        CUDA-event time of the n steps (ms) and the kernels per step."""
        out = (ctypes.c_int * max(1, int(n)))()
        ms = ctypes.c_float()
        nk = ctypes.c_int()
        check(self.lib.lumina_decode_greedy(self.h, int(token), int(n), out,
                                            ctypes.byref(ms) if timed else None,
                                            ctypes.byref(nk) if timed else None), self.lib)
        toks = list(out)[:int(n)]
        return (toks, ms.value, nk.value) if timed else toks

    def profile_attention(self, iters: int = 4):
        """Device time of the decode row's attention of every layer at the
        current KV length, replayed alone in a CUDA graph: (ms per launch,
        algorithmic bytes per launch)."""
        ms = ctypes.c_float()
        by = ctypes.c_double()
        check(self.lib.lumina_profile_attention(self.h, int(iters), ctypes.byref(ms), ctypes.byref(by)), self.lib)
        return ms.value, by.value

    def profile_gemv(self, iters: int = 4):
        """Device time of the decode token's packed GEMVs, replayed alone in a
        CUDA graph: (ms per launch, launches per token, algorithmic bytes per
        token = packed codes + scales + activations in + outputs)."""
        ms = ctypes.c_float()
        nl = ctypes.c_int()
        by = ctypes.c_double()
        check(self.lib.lumina_profile_gemv(self.h, int(iters), ctypes.byref(ms), ctypes.byref(nl),
                                           ctypes.byref(by)), self.lib)
        return ms.value, nl.value, by.value


# ---------------------------------------------------------------------------
# host sampler (chat.py:330-378), unchanged semantics
# ---------------------------------------------------------------------------
def make_pick(temperature=0.0, top_p=1.0, top_k=0, min_p=0.0, typical_p=1.0, repeat_penalty=1.0, rng=None):
    rng = rng if rng is not None else np.random.default_rng(0)

    def greedy_only():
        return temperature <= 0 and top_k <= 1 and min_p <= 0 and typical_p >= 1.0 and repeat_penalty == 1.0

    fast_greedy = greedy_only()

    def pick(lg, seen):
        if fast_greedy:
            # no penalty and no sampling: the argmax of the logits as given
            # (widening to float64 first, as below, is exact and keeps the
            # order, so the first maximum is the same index)
            return int(np.argmax(lg))
        lg = np.asarray(lg, dtype=np.float64)
        if repeat_penalty != 1.0 and seen:
            lg = lg.copy()
            for t in set(seen[-64:]):
                if 0 <= t < lg.size:
                    lg[t] = lg[t] / repeat_penalty if lg[t] > 0 else lg[t] * repeat_penalty
        if temperature <= 0 and top_k <= 1 and min_p <= 0 and typical_p >= 1.0:
            return int(np.argmax(lg))
        z = (lg - lg.max()) / max(temperature if temperature > 0 else 1.0, 1e-6)
        p = np.exp(z)
        p = p / p.sum()
        if top_k and top_k > 0:
            keep = np.zeros_like(p, dtype=bool)
            keep[np.argpartition(-p, min(top_k, p.size - 1))[:top_k]] = True
            p = np.where(keep, p, 0.0)
            p = p / p.sum()
        if min_p > 0:
            keep = p >= (p.max() * min_p)
            keep[int(np.argmax(p))] = True
            p = np.where(keep, p, 0.0)
            p = p / p.sum()
        if top_p < 1.0:
            n = int(np.searchsorted(np.cumsum(np.sort(p)[::-1]), top_p)) + 1
            n = max(1, min(n, p.size))
            keep = np.zeros_like(p, dtype=bool)
            keep[np.argpartition(-p, n - 1)[:n]] = True
            p = np.where(keep, p, 0.0)
            p = p / p.sum()
        if typical_p < 1.0:
            ent = float(-(p * np.log(p + 1e-12)).sum())
            dev = np.abs(-np.log(p + 1e-12) - ent)
            order = np.argsort(dev, kind="stable")
            cum = np.cumsum(p[order])
            keep = np.zeros_like(p, dtype=bool)
            keep[order[cum <= typical_p]] = True
            keep[order[0]] = True
            p = np.where(keep, p, 0.0)
            p = p / p.sum()
        if temperature <= 0:
            return int(np.argmax(p))
        return int(rng.choice(p.size, p=p)) if p.size < 256 else int(np.argmax(rng.multinomial(1, p)))

    pick.greedy = greedy_only()
    return pick


def _decode_loop(model, first_logits, ids, out, max_tokens, t0, budget_s, stop_ids, pick, on_token):
    """The per-token loop of generate / generate_cached (chat.py:383-403,
    524-544) with each step one graph replay on the device."""
    lg = first_logits
    steps = 0
    while len(out) < max_tokens and time.perf_counter() - t0 < budget_s:
        nxt = pick(lg, ids + out)
        if nxt in stop_ids:
            break
        out.append(nxt)
        steps += 1
        if on_token is not None:
            try:
                on_token(nxt)
            except Exception:  # noqa: BLE001
                pass
        if len(out) >= max_tokens:
            # the reference runs the layers for the last token too; its KV
            # row is part of the state a later turn reuses
            model.decode_step(nxt, want_logits=False)
            break
        lg, _ = model.decode_step(nxt)
    return steps


def generate(model: CudaChatModel, prompt, max_tokens: int = 32, budget_s: float = 300.0,
             stop_ids: tuple = (151643,), rng=None, temperature: float = 0.0, top_p: float = 1.0,
             top_k: int = 0, min_p: float = 0.0, typical_p: float = 1.0, repeat_penalty: float = 1.0,
             on_token=None) -> dict:
    """chat.generate (chat.py:307-407) on the device: prefill, then one graph
    replay per token; the host keeps the sampler."""
    t0 = time.perf_counter()
    ids = model.tok.encode(prompt)
    pick = make_pick(temperature, top_p, top_k, min_p, typical_p, repeat_penalty, rng)
    model.kv_truncate(0)
    lg = model.forward(ids, 0)[0]
    out: list[int] = []
    steps = _decode_loop(model, lg, ids, out, max_tokens, t0, budget_s, stop_ids, pick, on_token)
    dt = time.perf_counter() - t0
    return {"text": model.tok.decode(out), "tokens": out,
            "tokens_per_second": len(out) / dt if dt else 0.0, "seconds": dt,
            "stats": {"steps": steps, "spec_accepted": 0, "spec_drafted": 0}}


def _common_prefix(a, b):
    n = min(len(a), len(b))
    i = 0
    while i < n and a[i] == b[i]:
        i += 1
    return i


def generate_cached(model: CudaChatModel, prompt, max_tokens: int = 32, budget_s: float = 300.0,
                    stop_ids: tuple = (151643,), rng=None, temperature: float = 0.0, top_p: float = 1.0,
                    top_k: int = 0, min_p: float = 0.0, typical_p: float = 1.0,
                    repeat_penalty: float = 1.0, on_token=None, state: dict | None = None) -> dict:
    """chat.generate_cached (chat.py:418-551): longest-common-prefix reuse of
    the device KV, truncation on divergence (a block-table length edit), and
    the fully-cached case replays the last prompt row at its own position."""
    t0 = time.perf_counter()
    ids = model.tok.encode(prompt)
    pick = make_pick(temperature, top_p, top_k, min_p, typical_p, repeat_penalty, rng)
    st = state if state is not None else {"ids": [], "kv": model.kv, "pos": 0}
    if st.get("kv") is not model.kv or model.kv_length() < st["pos"]:
        # a fresh state (or one whose rows another call dropped) owns no rows
        st["kv"] = model.kv
        st["ids"], st["pos"] = [], 0
    if model.kv_length() != st["pos"]:
        # rows past the state's history belong to some other call
        model.kv_truncate(st["pos"])
    common = _common_prefix(st["ids"], ids)
    if common < len(st["ids"]):
        model.kv_truncate(common)
        st["ids"] = st["ids"][:common]
        st["pos"] = common
    reused = len(st["ids"])
    delta = ids[len(st["ids"]):]
    pos = st["pos"]
    if len(delta):
        lg = model.forward(delta, pos)[0]
        pos += len(delta)
    else:
        # the reference replays the last row on a truncated copy (chat.py:
        # 454-467); re-appending that row at position pos-1 writes the same
        # K/V the live cache holds, so truncate-and-replay is equivalent
        pos0r = max(pos - 1, 0)
        model.kv_truncate(pos0r)
        lg = model.forward([ids[-1]], pos0r)[0]
    out: list[int] = []
    steps = _decode_loop(model, lg, ids, out, max_tokens, t0, budget_s, stop_ids, pick, on_token)
    pos = model.kv_length()
    st["ids"] = list(ids) + out
    st["pos"] = pos
    dt = time.perf_counter() - t0
    return {"text": model.tok.decode(out), "tokens": out,
            "tokens_per_second": len(out) / dt if dt else 0.0, "seconds": dt,
            "stats": {"steps": steps, "prefill_reused": reused, "prefill_computed": len(delta)},
            "cache_state": st}


# ---------------------------------------------------------------------------
# prompt-lookup speculative decoding (chat.py:553-648)
# ---------------------------------------------------------------------------
def pld_draft(ids: list, n: int = 4, gram: int = 3) -> list:
    """The continuation of the latest earlier occurrence of the last ``gram``
    tokens, up to ``n`` tokens; [] when there is none (chat.py:553-569)."""
    if len(ids) < gram + 1:
        return []
    key = ids[-gram:]
    for i in range(len(ids) - gram - 1, -1, -1):
        if ids[i:i + gram] == key:
            cont = ids[i + gram:i + gram + n]
            if cont:
                return cont
    return []


def _spec_stats(drafted, accepted, target_forwards, tokens_out):
    """SpecStats.as_dict (spec.py:26-53) for the counters this driver keeps."""
    return {"drafted": drafted, "accepted": accepted,
            "acceptance_rate": accepted / drafted if drafted else 0.0,
            "tokens_per_target_forward": tokens_out / target_forwards if target_forwards else 0.0,
            "target_forwards": target_forwards, "draft_forwards": 0, "tokens_out": tokens_out,
            "seconds_draft": 0.0, "seconds_verify": 0.0}


def generate_spec(model: CudaChatModel, prompt, max_tokens: int = 32, budget_s: float = 300.0,
                  stop_ids: tuple = (151643,), draft_n: int = 4, rng=None) -> dict:
    """chat.generate_spec (chat.py:572-648) on the device: prompt-lookup
    drafts verified by one multi-row forward (the draft rows' logits come
    back from the device), greedy acceptance, and the rollback of
    chat.py:636-638 as a KV truncation (a block-table length edit) before the
    bonus token's single-row forward. Replaces the reference driver, whose
    ``cache`` is a numpy dict; tokens and accounting are the reference's."""
    t0 = time.perf_counter()
    drafted_n = accepted_n = forwards = tokens_out = 0
    ids = model.tok.encode(prompt)
    model.kv_truncate(0)
    h_lg = model.forward(ids, 0)[0]
    pos, out = len(ids), []
    while len(out) < max_tokens and time.perf_counter() - t0 < budget_s:
        drafted = pld_draft(ids + out, draft_n)
        if not drafted:
            nxt = int(np.argmax(h_lg))
            if nxt in stop_ids:
                break
            out.append(nxt)
            h_lg, _ = model.decode_step(nxt)
            h_lg = h_lg.copy()
            pos += 1
            forwards += 1
            tokens_out += 1
            continue
        drafted_n += len(drafted)
        t_lg = model.forward(drafted, pos, all_rows=True)
        forwards += 1
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
            if a in stop_ids:
                out.append(a)
                dt = time.perf_counter() - t0
                return {"text": model.tok.decode(out), "tokens": out,
                        "spec": _spec_stats(drafted_n, accepted_n, forwards, tokens_out),
                        "tokens_per_second": len(out) / dt if dt else 0.0, "seconds": dt}
            out.append(a)
        model.kv_truncate(pos + len(acc))
        h_lg = model.forward([bonus], pos + len(acc))[0]
        forwards += 1
        pos += len(acc) + 1
    dt = time.perf_counter() - t0
    out = out[:max_tokens]
    return {"text": model.tok.decode(out), "tokens": out,
            "spec": _spec_stats(drafted_n, accepted_n, forwards, tokens_out),
            "tokens_per_second": len(out) / dt if dt else 0.0, "seconds": dt}


# ---------------------------------------------------------------------------
# tree verification (eagle.py:259-357, spec.py:56-83)
# ---------------------------------------------------------------------------
def build_tree_mask(parents):
    """spec.py:56-83: 0 where node i may attend node j (itself, ancestors)."""
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


def verify_tree(model: CudaChatModel, pos: int, tree_ids, parents, depths):
    """One forward over the children (depth >= 1) with the ancestry bias and
    true positions Lp-1+depth (eagle.py:259-291). Appends the children's K/V
    after the live rows (length pos); returns their logits in tree order."""
    order = [i for i in range(len(tree_ids)) if depths[i] >= 1]
    N = len(order)
    Lp = pos
    if model.kv_length() != Lp:
        raise LuminaError(5, "verify_tree: KV length %d != pos %d" % (model.kv_length(), Lp))
    tm = build_tree_mask(parents)
    bias = np.full((N, Lp + N), -np.inf, dtype=np.float32)
    bias[:, :Lp] = 0.0
    gidx = {old: new for new, old in enumerate(order)}
    for ni, oi in enumerate(order):
        for oj in range(len(parents)):
            if tm[oi, oj] == 0.0 and oj != 0 and oj in gidx:
                bias[ni, Lp + gidx[oj]] = 0.0
    pos_ov = np.array([Lp - 1 + depths[i] for i in order], dtype=np.int32)
    logits = model.forward([tree_ids[i] for i in order], Lp, all_rows=True, pos_override=pos_ov,
                           attn_bias=bias)
    return logits, order


def commit_verified(model: CudaChatModel, pos: int, toks, parents, depths, cur_lg_fn, max_tokens, out,
                    stop_ids=()):
    """eagle.py:294-357: greedy walk, then the accepted children's KV rows are
    gathered into path order on the device and the bonus token takes one
    standard forward. Returns (done, pos, logits of the new last row, last)."""
    accepted, cur, path = [], 0, []
    while True:
        top = int(np.argmax(cur_lg_fn(cur)))
        kids = [i for i in range(1, len(toks)) if parents[i] == cur]
        nxt = next((i for i in kids if toks[i] == top), None)
        accepted.append(top if nxt is None else toks[nxt])
        if nxt is None:
            break
        path.append(nxt)
        cur = nxt
    done = False
    for a in accepted:
        out.append(a)
        if a in stop_ids or len(out) >= max_tokens:
            done = True
            break
    order = [i for i in range(len(toks)) if depths[i] >= 1]
    gidx = {old: new for new, old in enumerate(order)}
    if done:
        model.kv_truncate(pos)
        return True, pos, None, out[-1]
    model.kv_commit_rows(pos, [gidx[i] for i in path])
    pos += len(path)
    lg = model.forward([accepted[-1]], pos)[0]
    return False, pos + 1, lg, accepted[-1]


# ---------------------------------------------------------------------------
# several sequences over one shared prefix (no reference counterpart: the
# reference serves one sequence per generate call and reuses a prefix
# through its prefix cache, chat.py:418-551)
# ---------------------------------------------------------------------------
def generate_shared_prefix(model: CudaChatModel, prefix_ids, suffixes, max_tokens: int = 32,
                           stop_ids: tuple = (), timed: bool = False):
    """Greedy decode of B sequences ``prefix_ids + suffixes[b]`` that share
    the prefix's KV rows on the device. The prefix is prefilled once; the
    suffixes go in forwards of up to 64 rows, and every decode step is one
    forward of the B (<= 64) live sequences' rows. Rows of all sequences
    live in the one KV cache side by side; each row attends to the prefix
    and to its own sequence's rows only (an additive -inf bias on the
    others, the tree-verification forward of ``verify_tree``) at its own
    true position, so sequence b sees exactly what ``generate(prefix +
    suffixes[b])`` would. ``max_tokens`` >= 1 tokens per sequence.

    Returns ``{"tokens": [list per sequence], "first_logits": (B, vocab)}``
    (the logits after each full prompt); with ``timed`` also the wall time of
    the decode steps ("decode_s") and the number of steps."""
    prefix = [int(t) for t in prefix_ids]
    sfx = [[int(t) for t in s] for s in suffixes]
    B = len(sfx)
    if B < 1 or any(len(s) < 1 for s in sfx) or not prefix:
        raise LuminaError(1, "generate_shared_prefix: a non-empty prefix and non-empty suffixes are needed")
    if max_tokens < 1:
        raise LuminaError(1, "generate_shared_prefix: max_tokens %d, at least 1" % max_tokens)
    chunk = min(64, model.max_rows)  # rows of one biased forward (the library's bias buffer holds 64)
    if B > chunk:
        raise LuminaError(1, "generate_shared_prefix: %d sequences, at most %d" % (B, chunk))
    P = len(prefix)
    model.kv_truncate(0)
    model.forward(prefix, 0)
    rows = [[] for _ in range(B)]  # KV rows of each sequence after the prefix
    pos = [P] * B                  # next position of each sequence

    def step(toks_per_seq, live):
        """One forward of the given rows: live[i] is the sequence of row i.
        A row admits the prefix, its sequence's cached rows (bias +1: their
        cache index can exceed the row's position) and its sequence's rows
        of this forward up to itself; every other key gets -inf."""
        T = model.kv_length()
        n = len(live)
        bias = np.full((n, T + n), -np.inf, dtype=np.float32)
        bias[:, :P] = 0.0
        po = np.empty(n, np.int32)
        for i, b in enumerate(live):
            if rows[b]:
                bias[i, rows[b]] = 1.0
        for i, b in enumerate(live):
            rows[b].append(T + i)
            po[i] = pos[b]
            pos[b] += 1
            bias[i, [T + j for j in range(i + 1) if live[j] == b]] = 0.0
        return model.forward(list(toks_per_seq), T, all_rows=True, pos_override=po, attn_bias=bias)

    # the suffixes: forwards of up to `chunk` rows, causal within a suffix
    # (a later chunk sees its sequences' earlier rows as cached rows)
    live = [b for b in range(B) for _ in sfx[b]]
    toks = [t for b in range(B) for t in sfx[b]]
    lg = np.concatenate([step(toks[c:c + chunk], live[c:c + chunk]) for c in range(0, len(toks), chunk)])
    ends = np.cumsum([len(s) for s in sfx]) - 1
    first_logits = lg[ends].copy()
    nxt = [int(np.argmax(first_logits[b])) for b in range(B)]
    out = [[] for _ in range(B)]
    done = [False] * B
    t0 = time.perf_counter()
    steps = 0
    while True:
        for b in range(B):
            if not done[b]:
                out[b].append(nxt[b])
                if nxt[b] in stop_ids or len(out[b]) >= max_tokens:
                    done[b] = True
        live = [b for b in range(B) if not done[b]]
        if not live:
            break
        lg = step([nxt[b] for b in live], live)
        steps += 1
        for i, b in enumerate(live):
            nxt[b] = int(np.argmax(lg[i]))
    res = {"tokens": out, "first_logits": first_logits}
    if timed:
        res["decode_s"] = time.perf_counter() - t0
        res["steps"] = steps
    return res
