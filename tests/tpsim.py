"""A numpy restatement of the engine's tensor-parallel split, for CPU tests.

Each rank holds the shard `smotor.tp_plan` assigns it (query/KV heads, FFN
columns, output-head rows), runs the qwen2/llama forward of
crates/s-models/src/qwen2.rs:460-561 on it in float64, and combines partial
results with the same collectives the engine uses: a sum over ranks after
attn_output and after ffn_down, and a gather of the logit slices. Weights are
the oracle's dequantization of the GGUF tensors (dequant.rs:209-310).
Test infrastructure only.
"""
import numpy as np

import pyoracle as orc
import smotor


class Gguf:
    def __init__(self, path):
        self.path = path
        self.info = orc.gguf_info(path)
        self.by_name = {t["name"]: t for t in self.info["tensors"]}
        self.raw = open(path, "rb").read()
        md = self.info["metadata"]
        arch = md["general.architecture"]["value"]
        g = lambda k: md[f"{arch}.{k}"]["value"]
        self.H, self.L = g("embedding_length"), g("block_count")
        self.Hq, self.Hkv, self.F = g("attention.head_count"), g("attention.head_count_kv"), g("feed_forward_length")
        self.theta, self.eps = np.float32(g("rope.freq_base")), np.float32(g("attention.layer_norm_rms_epsilon"))
        self.hd = self.H // self.Hq
        self.V = self.by_name["token_embd.weight"]["dims"][1]

    def has(self, name):
        return name in self.by_name

    def tensor(self, name):
        t = self.by_name[name]
        n = int(np.prod(t["dims"]))
        off = self.info["data_start"] + t["offset"]
        x = orc.dequantize(t["type"], n, self.raw[off:off + t["n_bytes"]]).astype(np.float64)
        return x.reshape(t["dims"][::-1]) if len(t["dims"]) == 2 else x

    def config(self):
        return smotor.config_of(self.L, self.H, self.F, self.Hq, self.Hkv, self.V, float(self.theta), float(self.eps))


def rmsnorm(x, w, eps):
    return x * (1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)) * w


def rope(x, pos0, theta, hd):
    """NEOX half-split rotation of [S, heads, hd] (qwen2.rs:708-724)."""
    half = hd // 2
    i = np.arange(half, dtype=np.float32)
    freq = np.power(np.float32(theta), -(np.float32(2.0) * i) / np.float32(hd)).astype(np.float32)
    pos = (np.arange(x.shape[0]) + pos0).astype(np.float32)
    ang = (pos[:, None] * freq[None, :]).astype(np.float32)
    c, s = np.cos(ang)[:, None, :].astype(np.float64), np.sin(ang)[:, None, :].astype(np.float64)
    a, b = x[..., :half], x[..., half:]
    return np.concatenate([a * c - b * s, a * s + b * c], axis=-1)


def forward(g: Gguf, tokens, rank, world, all_reduce, all_gather):
    """Logits of the last token for a prefill of `tokens` at position 0 on
    this rank's shard; all_reduce(sum) / all_gather(list) are the
    collectives between ranks."""
    sh = smotor.tp_plan(g.config(), rank, world)
    hd, G = g.hd, g.Hq // g.Hkv
    qs = slice(sh.q_head0 * hd, (sh.q_head0 + sh.q_heads) * hd)
    ks = slice(sh.kv_head0 * hd, (sh.kv_head0 + sh.kv_heads) * hd)
    fs = slice(sh.ff0, sh.ff0 + sh.ff)
    emb = g.tensor("token_embd.weight")
    x = emb[np.asarray(tokens)]
    S = x.shape[0]
    for li in range(g.L):
        p = f"blk.{li}."
        xn = rmsnorm(x, g.tensor(p + "attn_norm.weight"), g.eps)
        proj = {}
        for n, sl in (("q", qs), ("k", ks), ("v", ks)):
            y = xn @ g.tensor(p + f"attn_{n}.weight")[sl].T
            if g.has(p + f"attn_{n}.bias"):
                y = y + g.tensor(p + f"attn_{n}.bias")[sl]
            proj[n] = y
        q = rope(proj["q"].reshape(S, sh.q_heads, hd), 0, g.theta, hd)
        k = rope(proj["k"].reshape(S, sh.kv_heads, hd), 0, g.theta, hd)
        v = proj["v"].reshape(S, sh.kv_heads, hd)
        att = np.empty((S, sh.q_heads, hd))
        for h in range(sh.q_heads):
            kvh = h // G  # GQA within the shard: whole groups stay together
            sc = (q[:, h] @ k[:, kvh].T) * (1.0 / np.sqrt(hd))
            sc = np.where(np.tril(np.ones((S, S), bool)), sc, -np.inf)
            w = np.exp(sc - sc.max(-1, keepdims=True))
            w /= w.sum(-1, keepdims=True)
            att[:, h] = w @ v[:, kvh]
        o = att.reshape(S, -1) @ g.tensor(p + "attn_output.weight")[:, qs].T
        x = x + all_reduce(o)
        xn = rmsnorm(x, g.tensor(p + "ffn_norm.weight"), g.eps)
        gt = xn @ g.tensor(p + "ffn_gate.weight")[fs].T
        up = xn @ g.tensor(p + "ffn_up.weight")[fs].T
        h_ = gt / (1.0 + np.exp(-gt)) * up
        x = x + all_reduce(h_ @ g.tensor(p + "ffn_down.weight")[:, fs].T)
    xn = rmsnorm(x[-1], g.tensor("output_norm.weight"), g.eps)
    head = g.tensor("output.weight") if g.has("output.weight") else emb
    part = head[sh.vocab0:sh.vocab0 + sh.vocab] @ xn
    return np.concatenate(all_gather(part))
