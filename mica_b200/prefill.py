"""Prefill scorer for a dense Qwen3-style decoder on the W8A8 kernels.

This is the model-level caller of the hot path: it restates what the reference's
PrefillEngine does for one request (v0.5/serving/lib/prefill_engine.py:274-339 run /
final_hidden, :385-418 capture / replay) on the dense decoder of BASELINE configs 3-4
(Qwen3-4B dims: hidden 2560, 32 q / 8 kv heads x 128, FFN 9728, 36 layers).

Per layer, seven launches of this library plus attention:
  rmsnorm_quant(prev_out, residual)  -> new residual stream + int8 codes (fused prologue)
  w8a8 GEMM QKV (tcgen05)            -> q, k, v
  qk_norm_rope                       -> q/k RMSNorm + RoPE in place (the HF op sequence)
  attention: torch SDPA (cuDNN/flash), causal, GQA
  act_quant(attn) + w8a8 GEMM O
  rmsnorm_quant(o, residual)         -> codes for the MLP
  gate_up GEMM + SwiGLU + requant    -> codes for down (one cooperative launch)
  w8a8 GEMM down
Models with per-projection smoothing (an int8-w8a8/1 file, load_model) quantise a block's
normed input once per distinct smoothing vector and, when gate and up differ, run them as
two GEMMs plus one SwiGLU + requant kernel.
The last layer computes K/V for every row but Q, attention, O and the MLP only for the
scored row (prefill_engine.py:306-339), then the fused final norm + gathered lm_head GEMV
+ option softmax (release_runtime.py:302-306, :509-522).

Graphs: capture() records the whole prefill for a 64-token bucket with a static id
buffer and a `limit` row (the real length), like the reference's per-bucket graphs; rows
past `limit` are padding that no real row attends to. capture_batch() does the same for a
padded [B, L] batch (per-request limits and option slices), like the reference's batch graphs.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import _native as N
from . import int8_kernels as K
from . import ops  # noqa: F401
from .int8_runtime import InvalidModel, interleave_gate_up, quant_weight, read_int8_file

BUCKET = 64            # graph buckets (the reference's 64-token buckets)
EAGER_BUCKET = 256     # padding granularity of eager (uncaptured) requests


@dataclass
class DecoderConfig:
    hidden: int = 2560
    inter: int = 9728
    layers: int = 36
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    vocab: int = 151936
    eps: float = 1e-6
    rope_theta: float = 1e6
    tie_embeddings: bool = True

    @property
    def q_dim(self):
        return self.heads * self.head_dim

    @property
    def kv_dim(self):
        return self.kv_heads * self.head_dim


@dataclass
class Layer:
    """One decoder layer's weights. int8 weights [N, K] with fp32 channel scales [N];
    optional fp32 biases [N] and smoothing vectors inv_smooth [K] (the reference QLinear's
    buffers, lib/int8_runtime.py:108-127).

    q/k/v are stacked into qkv_w. qkv_parts lists the row ranges (lo, hi, inv) that share one
    input quantisation: one part when the three projections quantise x alike (no smoothing,
    or the same inv_smooth), else one part per projection. The MLP is fused (gu_w/gu_s:
    gate and up rows interleaved by interleave_gate_up, sharing inv gu_inv) or, when gate and
    up are smoothed differently, split (g_* and u_* kept apart)."""
    in_norm: torch.Tensor
    qkv_w: torch.Tensor
    qkv_s: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    o_w: torch.Tensor
    o_s: torch.Tensor
    post_norm: torch.Tensor
    gu_w: torch.Tensor
    gu_s: torch.Tensor
    down_w: torch.Tensor
    down_s: torch.Tensor
    qkv_b: torch.Tensor = None
    qkv_parts: list = None          # [(lo, hi, inv or None)]; None = one part, no smoothing
    o_inv: torch.Tensor = None
    o_b: torch.Tensor = None
    gu_inv: torch.Tensor = None
    gu_b: torch.Tensor = None
    split_mlp: tuple = None         # (g_w, g_s, g_inv, g_b, u_w, u_s, u_inv, u_b) when gu_w is None
    down_inv: torch.Tensor = None
    down_b: torch.Tensor = None

    def parts(self):
        return self.qkv_parts if self.qkv_parts is not None else [(0, self.qkv_w.shape[0], None)]

    def mlp_in_inv(self):
        """Smoothing of the MLP's first quantisation (gate's when split)."""
        return self.split_mlp[2] if self.split_mlp is not None else self.gu_inv

    def distinct_attn_invs(self) -> int:
        return len({_inv_key(inv) for _, _, inv in self.parts()})

    def distinct_mlp_invs(self) -> int:
        return 1 if self.split_mlp is None else len({_inv_key(self.split_mlp[2]), _inv_key(self.split_mlp[6])})


def _inv_key(inv):
    return None if inv is None else inv.data_ptr()


@dataclass
class Decoder:
    cfg: DecoderConfig
    embed: torch.Tensor                      # bf16 [vocab, hidden]
    layers: list = field(default_factory=list)
    final_norm: torch.Tensor = None          # bf16 [hidden]
    lm_head: torch.Tensor = None             # bf16 [vocab, hidden] (None = tied to embed)

    @property
    def device(self):
        return self.embed.device


# ---------------------------------------------------------------------------------------
def _q(w):
    q, s = quant_weight(w)
    return q.contiguous(), s.contiguous()


def from_hf_state(state: dict, cfg: DecoderConfig, device) -> Decoder:
    """Builds the decoder from a HF Qwen3ForCausalLM state dict (bf16), quantising every
    projection per output row exactly as the reference's QLinear does (no smoothing)."""
    def t(name):
        return state[name].to(device)

    layers = []
    for i in range(cfg.layers):
        p = f'model.layers.{i}.'
        qkv = torch.cat([t(p + 'self_attn.q_proj.weight'), t(p + 'self_attn.k_proj.weight'),
                         t(p + 'self_attn.v_proj.weight')]).float()
        qkv_w, qkv_s = _q(qkv)
        o_w, o_s = _q(t(p + 'self_attn.o_proj.weight').float())
        g_w, g_s = _q(t(p + 'mlp.gate_proj.weight').float())
        u_w, u_s = _q(t(p + 'mlp.up_proj.weight').float())
        d_w, d_s = _q(t(p + 'mlp.down_proj.weight').float())
        layers.append(Layer(
            in_norm=t(p + 'input_layernorm.weight').to(torch.bfloat16).contiguous(),
            qkv_w=qkv_w, qkv_s=qkv_s,
            q_norm=t(p + 'self_attn.q_norm.weight').to(torch.bfloat16).contiguous(),
            k_norm=t(p + 'self_attn.k_norm.weight').to(torch.bfloat16).contiguous(),
            o_w=o_w, o_s=o_s,
            post_norm=t(p + 'post_attention_layernorm.weight').to(torch.bfloat16).contiguous(),
            gu_w=interleave_gate_up(g_w, u_w), gu_s=interleave_gate_up(g_s, u_s),
            down_w=d_w, down_s=d_s))
    lm = state.get('lm_head.weight')
    return Decoder(cfg=cfg, embed=t('model.embed_tokens.weight').to(torch.bfloat16).contiguous(), layers=layers,
                   final_norm=t('model.norm.weight').to(torch.bfloat16).contiguous(),
                   lm_head=None if (lm is None or cfg.tie_embeddings) else lm.to(device).to(torch.bfloat16))


# ---- INT8 weights file ------------------------------------------------------------------
_ATTN = ('q_proj', 'k_proj', 'v_proj', 'o_proj')
_MLP = ('gate_proj', 'up_proj', 'down_proj')


def config_from_hf(d: dict) -> DecoderConfig:
    """DecoderConfig from a HF Qwen3 config.json dictionary."""
    heads = d['num_attention_heads']
    return DecoderConfig(hidden=d['hidden_size'], inter=d['intermediate_size'], layers=d['num_hidden_layers'],
                         heads=heads, kv_heads=d.get('num_key_value_heads', heads),
                         head_dim=d.get('head_dim') or d['hidden_size'] // heads, vocab=d['vocab_size'],
                         eps=d.get('rms_norm_eps', 1e-6), rope_theta=d.get('rope_theta', 1e6),
                         tie_embeddings=d.get('tie_word_embeddings', True))


def config_from_int8(t: dict, ties: dict) -> DecoderConfig:
    """DecoderConfig inferred from the tensors of an int8-w8a8/1 file (eps and rope theta take
    the Qwen3 defaults)."""
    p = 'model.layers.0.'
    try:
        vocab, hidden = t['model.embed_tokens.weight'].shape
        head_dim = t[p + 'self_attn.q_norm.weight'].numel()
        q_dim = t[p + 'self_attn.q_proj.qweight'].shape[0]
        kv_dim = t[p + 'self_attn.k_proj.qweight'].shape[0]
        inter = t[p + 'mlp.gate_proj.qweight'].shape[0]
    except KeyError as e:
        raise InvalidModel(f'not a dense Qwen3 decoder: {e.args[0]} missing') from None
    layers = 1 + max(int(k.split('.')[2]) for k in t if k.startswith('model.layers.'))
    return DecoderConfig(hidden=hidden, inter=inter, layers=layers, heads=q_dim // head_dim,
                         kv_heads=kv_dim // head_dim, head_dim=head_dim, vocab=vocab,
                         tie_embeddings='lm_head.weight' in ties or 'lm_head.weight' not in t)


def _expected(cfg: DecoderConfig):
    """key -> (dtype, shape) of every tensor a dense Qwen3 decoder file holds; the QLinear
    keys inv_smooth and bias are optional (reported separately)."""
    bf, H, D = torch.bfloat16, cfg.hidden, cfg.head_dim
    dims = {'q_proj': (cfg.q_dim, H), 'k_proj': (cfg.kv_dim, H), 'v_proj': (cfg.kv_dim, H),
            'o_proj': (H, cfg.q_dim), 'gate_proj': (cfg.inter, H), 'up_proj': (cfg.inter, H),
            'down_proj': (H, cfg.inter)}
    need = {'model.embed_tokens.weight': (bf, (cfg.vocab, H)), 'model.norm.weight': (bf, (H,)),
            'lm_head.weight': (bf, (cfg.vocab, H))}
    opt = {}
    for i in range(cfg.layers):
        p = f'model.layers.{i}.'
        for n in ('input_layernorm', 'post_attention_layernorm'):
            need[p + n + '.weight'] = (bf, (H,))
        for n in ('q_norm', 'k_norm'):
            need[p + 'self_attn.' + n + '.weight'] = (bf, (D,))
        for grp, names in (('self_attn.', _ATTN), ('mlp.', _MLP)):
            for n in names:
                o, k = dims[n]
                q = p + grp + n
                need[q + '.qweight'] = (torch.int8, (o, k))
                need[q + '.wscale'] = (torch.float32, (o,))
                opt[q + '.inv_smooth'] = (torch.float32, (k,))
                opt[q + '.bias'] = (torch.float32, (o,))
    return need, opt


def from_int8_state(t: dict, cfg: DecoderConfig, device) -> Decoder:
    """Builds the decoder from the tensors of an int8-w8a8/1 file: the stored int8 weights,
    channel scales, smoothing vectors and biases are used as they are (no requantisation).
    Projections whose input quantisation matches are stacked (q|k|v) or interleaved
    (gate|up) for the fused kernels; differently smoothed ones stay apart."""
    need, opt = _expected(cfg)
    missing = sorted(k for k in need if k not in t and not (k == 'lm_head.weight' and cfg.tie_embeddings))
    extra = sorted(k for k in t if k not in need and k not in opt)
    if missing or extra:
        raise InvalidModel(f'missing {missing[:4]} / unexpected {extra[:4]} (dense Qwen3 decoders only)')
    for k, v in t.items():
        dt, shape = need.get(k) or opt[k]
        if v.dtype != dt or tuple(v.shape) != shape:
            raise InvalidModel(f'{k}: {v.dtype} {tuple(v.shape)}, expected {dt} {shape}')

    def g(key):
        v = t.get(key)
        return None if v is None else v.to(device).contiguous()

    def proj(prefix):
        return g(prefix + '.qweight'), g(prefix + '.wscale'), g(prefix + '.inv_smooth'), g(prefix + '.bias')

    def cat_bias(ps):
        if all(b is None for *_, b in ps):
            return None
        return torch.cat([b if b is not None else torch.zeros_like(s) for _, s, _, b in ps]).contiguous()

    from .int8_runtime import same_smoothing
    layers = []
    for i in range(cfg.layers):
        p = f'model.layers.{i}.'
        qkv = [proj(p + 'self_attn.' + n) for n in ('q_proj', 'k_proj', 'v_proj')]
        bounds = [0, cfg.q_dim, cfg.q_dim + cfg.kv_dim, cfg.q_dim + 2 * cfg.kv_dim]
        invs = [x[2] for x in qkv]
        if same_smoothing(invs[0], invs[1]) and same_smoothing(invs[0], invs[2]):
            parts = None if invs[0] is None else [(0, bounds[3], invs[0])]
        else:
            parts = [(bounds[j], bounds[j + 1], invs[j]) for j in range(3)]
        o_w, o_s, o_inv, o_b = proj(p + 'self_attn.o_proj')
        gp, up, dp = (proj(p + 'mlp.' + n) for n in _MLP)
        lay = dict(in_norm=g(p + 'input_layernorm.weight'),
                   qkv_w=torch.cat([x[0] for x in qkv]).contiguous(), qkv_s=torch.cat([x[1] for x in qkv]).contiguous(),
                   qkv_b=cat_bias(qkv), qkv_parts=parts,
                   q_norm=g(p + 'self_attn.q_norm.weight'), k_norm=g(p + 'self_attn.k_norm.weight'),
                   o_w=o_w, o_s=o_s, o_inv=o_inv, o_b=o_b, post_norm=g(p + 'post_attention_layernorm.weight'),
                   down_w=dp[0], down_s=dp[1], down_inv=dp[2], down_b=dp[3])
        if same_smoothing(gp[2], up[2]):
            bias = None
            if gp[3] is not None or up[3] is not None:
                bias = interleave_gate_up(gp[3] if gp[3] is not None else torch.zeros_like(gp[1]),
                                          up[3] if up[3] is not None else torch.zeros_like(up[1]))
            lay.update(gu_w=interleave_gate_up(gp[0], up[0]), gu_s=interleave_gate_up(gp[1], up[1]),
                       gu_inv=gp[2], gu_b=bias)
        else:
            lay.update(gu_w=None, gu_s=None, split_mlp=(*gp, *up))
        layers.append(Layer(**lay))
    lm = t.get('lm_head.weight')
    embed = g('model.embed_tokens.weight')
    tied = lm is None or lm is t['model.embed_tokens.weight']
    return Decoder(cfg=cfg, embed=embed, layers=layers, final_norm=g('model.norm.weight'),
                   lm_head=None if tied else lm.to(device).contiguous())


def load_model(path, device, cfg: DecoderConfig = None) -> Decoder:
    """The reference's int8_runtime.load_model (lib/int8_runtime.py:665-726) for dense Qwen3
    decoders: reads model-int8.safetensors (a folder, with its config.json when present, or
    the file itself) and builds the Decoder on `device`."""
    import json
    from pathlib import Path
    path = Path(path)
    tensors, ties = read_int8_file(path)
    if cfg is None:
        cj = (path if path.is_dir() else path.parent) / 'config.json'
        cfg = config_from_hf(json.loads(cj.read_text())) if cj.is_file() else config_from_int8(tensors, ties)
    return from_int8_state(tensors, cfg, torch.device(device))


def random_decoder(cfg: DecoderConfig, device, seed: int = 0, std: float = 0.02) -> Decoder:
    """Random-init decoder of the given dims, generated on the device: bf16 weights N(0, std)
    quantised per output row (as converting a random-init HF model would), norm weights
    N(1, 0.1)."""
    g = torch.Generator(device=device).manual_seed(seed)
    H, I = cfg.hidden, cfg.inter

    def w(n, k):
        return _q(torch.randn(n, k, generator=g, device=device) * std)

    def gamma(n):
        return (1 + 0.1 * torch.randn(n, generator=g, device=device)).to(torch.bfloat16)

    layers = []
    for _ in range(cfg.layers):
        qkv_w, qkv_s = w(cfg.q_dim + 2 * cfg.kv_dim, H)
        o_w, o_s = w(H, cfg.q_dim)
        g_w, g_s = w(I, H)
        u_w, u_s = w(I, H)
        d_w, d_s = w(H, I)
        layers.append(Layer(in_norm=gamma(H), qkv_w=qkv_w, qkv_s=qkv_s, q_norm=gamma(cfg.head_dim),
                            k_norm=gamma(cfg.head_dim), o_w=o_w, o_s=o_s, post_norm=gamma(H),
                            gu_w=interleave_gate_up(g_w, u_w), gu_s=interleave_gate_up(g_s, u_s), down_w=d_w,
                            down_s=d_s))
        del g_w, u_w
    embed = (torch.randn(cfg.vocab, H, generator=g, device=device) * std).to(torch.bfloat16)
    return Decoder(cfg=cfg, embed=embed, layers=layers, final_norm=gamma(H))


# ---------------------------------------------------------------------------------------
def rope_tables(cfg: DecoderConfig, n: int, device):
    """cos/sin [n, head_dim] in bf16, computed in fp32 as HF Qwen3RotaryEmbedding does."""
    d = cfg.head_dim
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.int64, device=device).float() / d))
    pos = torch.arange(n, device=device).float()
    freqs = (inv[:, None] @ pos[None, :]).t()
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)


class _Normed:
    """A block's normed input, quantised once per distinct smoothing vector: the fused
    norm kernel's codes serve the first consumer, and the normed activations y (kept only
    when another consumer smooths differently) are requantised for the others."""

    def __init__(self, q, s, inv, y):
        self.m = q.shape[0]
        self.y = y
        self.cache = {_inv_key(inv): (q, s)}

    def codes(self, inv, rows=None):
        key = _inv_key(inv)
        if key not in self.cache:
            self.cache[key] = torch.ops.mica.act_quant(self.y, inv, K._round_code())
        q, s = self.cache[key]
        if rows is None:
            return q, s
        return q.index_select(0, rows), s.index_select(0, rows)


class Prefill:
    """Scores requests on a Decoder: ids -> option probabilities of the last position."""

    def __init__(self, model: Decoder, option_ids, max_len: int = 32768, attn_backends=None, attention: str = 'sdpa'):
        """attention: 'sdpa' runs the causal attention of the full-length layers through torch SDPA
        (cuDNN first, `attn_backends`); 'mica' runs it with this library's tcgen05 kernel
        (mica_attention_prefill), reading q/k/v in place from the QKV projection's output. The
        last layer's last-row attention uses SDPA either way."""
        if attention not in ('sdpa', 'mica'):
            raise ValueError(f"attention must be 'sdpa' or 'mica', not {attention!r}")
        if attention == 'mica' and model.cfg.head_dim != 128:
            raise ValueError(f"attention='mica' needs head_dim 128, not {model.cfg.head_dim}")
        self.attention = attention
        self.m = model
        cfg = model.cfg
        dev = model.device
        self.cfg = cfg
        head = model.lm_head if model.lm_head is not None else model.embed
        ids = torch.as_tensor(option_ids, device=dev, dtype=torch.long)
        self.rows = head.index_select(0, ids).float().contiguous()      # release_runtime.py:302
        self.cos, self.sin = rope_tables(cfg, max_len, dev)
        self.max_len = max_len
        self.scale = cfg.head_dim ** -0.5
        self.graphs = {}
        self.batch_graphs = {}
        self.pool = None
        self._pos = {}
        if attn_backends is None:
            from torch.nn.attention import SDPBackend
            attn_backends = [SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION]
        self.backends = attn_backends

    # ---- pieces ------------------------------------------------------------------------
    def _norm_quant(self, x, w, residual=None, inv=None, want_y=False):
        """Fused residual add + RMSNorm + quantisation of y * inv. Returns (q, s, residual
        stream, y); y (the normed activations) only when want_y."""
        q, s, y, summed = torch.ops.mica.rmsnorm_quant(x, residual, w, inv, self.cfg.eps, N.NORM_WEIGHT,
                                                        K._round_code(), want_y, True)
        return q, s, (summed if residual is not None else x), (y if want_y else None)

    def _normed(self, x, w, residual, inv0, n_inv):
        q, s, h, y = self._norm_quant(x, w, residual, inv0, want_y=n_inv > 1)
        return _Normed(q, s, inv0, y), h

    def _gemm(self, q, s, w, sw, bias=None):
        tile = K.gemm_tile(w.shape[0], w.shape[1], q.shape[0], q.device)
        return torch.ops.mica.w8a8_gemm(q, s, w, sw, bias, 0, tile)

    def _qkv_cols(self, lay, nq, lo, hi, rows=None):
        """Columns [lo, hi) of the q|k|v projection of the normed input `nq` (for `rows` only,
        when given), one GEMM per part that quantises the input differently."""
        parts = [(max(a, lo), min(b, hi), inv) for a, b, inv in lay.parts() if min(b, hi) > max(a, lo)]
        bias = lay.qkv_b
        if len(parts) == 1:
            a, b, inv = parts[0]
            q, s = nq.codes(inv, rows)
            return self._gemm(q, s, lay.qkv_w[a:b], lay.qkv_s[a:b], None if bias is None else bias[a:b])
        m = nq.m if rows is None else rows.numel()
        out = torch.empty((m, hi - lo), dtype=torch.bfloat16, device=lay.qkv_w.device)
        for a, b, inv in parts:
            q, s = nq.codes(inv, rows)
            w = lay.qkv_w[a:b]
            torch.ops.mica.w8a8_gemm_into(q, s, w, lay.qkv_s[a:b], None if bias is None else bias[a:b],
                                          out[:, a - lo:b - lo], K.gemm_tile(w.shape[0], w.shape[1], m, q.device))
        return out

    def _attention(self, q, k, v, causal, mask=None):
        """q [B, Sq, H, D], k/v [B, Sk, KV, D] (strided views are fine) -> [B*Sq, H*D]."""
        from torch.nn.attention import sdpa_kernel
        with sdpa_kernel(self.backends):
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                               attn_mask=mask, is_causal=causal and mask is None, scale=self.scale,
                                               enable_gqa=True)
        return o.transpose(1, 2).reshape(q.shape[0] * q.shape[1], -1).contiguous()

    def _mlp(self, nm, lay):
        """gate/up + SwiGLU + requant (down_proj's smoothing applied there), then down."""
        if lay.split_mlp is None:
            q, s = nm.codes(lay.gu_inv)
            _, qh, sh = torch.ops.mica.gemm_swiglu_quant(q, s, lay.gu_w, lay.gu_s, lay.gu_b, lay.down_inv,
                                                         K._round_code())
        else:
            g_w, g_s, g_inv, g_b, u_w, u_s, u_inv, u_b = lay.split_mlp
            g = self._gemm(*nm.codes(g_inv), g_w, g_s, g_b)
            u = self._gemm(*nm.codes(u_inv), u_w, u_s, u_b)
            _, qh, sh = torch.ops.mica.swiglu_quant(g, u, lay.down_inv, K._round_code(), False, True)
        return self._gemm(qh, sh, lay.down_w, lay.down_s, lay.down_b)

    def _positions(self, B, L, device):
        """Row positions of a [B, L] batch (None for B = 1: the kernel uses the row index)."""
        if B == 1:
            return None
        key = (B, L)
        if key not in self._pos:
            self._pos[key] = torch.arange(L, device=device, dtype=torch.long).repeat(B)
        return self._pos[key]

    # ---- forward -------------------------------------------------------------------------
    def hidden_last(self, ids: torch.Tensor, limit: torch.Tensor = None, last_only: bool = True):
        """Runs the decoder over ids [S] (one request) or [B, L] (B requests padded to L) and
        returns each request's last real row's hidden state (before the final norm) as bf16
        [B, hidden]. `limit` (int64 [B]) is each request's real length when padded; keys at
        or past it are masked for the scored row, and no real row attends to later rows."""
        cfg, m = self.cfg, self.m
        if ids.dim() == 1:
            ids = ids[None]
        B, L = ids.shape
        M = B * L
        pos = self._positions(B, L, ids.device)
        h = F.embedding(ids.reshape(-1), m.embed)
        prev = None
        nl = len(m.layers)
        for li, lay in enumerate(m.layers):
            nq, h = self._normed(prev if prev is not None else h, lay.in_norm, h if prev is not None else None,
                                 lay.parts()[0][2], lay.distinct_attn_invs())
            if li == nl - 1 and last_only:
                return self._last_layer(nq, h, lay, B, L, pos, limit)
            qkv = self._qkv_cols(lay, nq, 0, lay.qkv_w.shape[0])
            torch.ops.mica.qk_norm_rope(qkv, lay.q_norm, lay.k_norm, self.cos, self.sin, pos, 0, cfg.heads,
                                        cfg.kv_heads, cfg.eps)
            if self.attention == 'mica':
                # each request attends causally within its own L rows; padding rows sit after a
                # request's real rows, so no real row sees them
                attn = torch.ops.mica.attention_prefill(qkv, B, L, cfg.heads, cfg.kv_heads, self.scale)
            else:
                q, k, v = qkv.split([cfg.q_dim, cfg.kv_dim, cfg.kv_dim], dim=1)
                attn = self._attention(q.view(B, L, cfg.heads, cfg.head_dim), k.view(B, L, cfg.kv_heads, cfg.head_dim),
                                       v.view(B, L, cfg.kv_heads, cfg.head_dim), causal=True)
            qa, sa = torch.ops.mica.act_quant(attn, lay.o_inv, K._round_code())
            o = self._gemm(qa, sa, lay.o_w, lay.o_s, lay.o_b)
            nm, h = self._normed(o, lay.post_norm, h, lay.mlp_in_inv(), lay.distinct_mlp_invs())
            prev = self._mlp(nm, lay)
        out = h + prev
        return out.index_select(0, self._scored_rows(B, L, limit, out.device))

    def _scored_rows(self, B, L, limit, device):
        base = torch.arange(B, device=device, dtype=torch.long) * L
        return base + ((limit.view(B) - 1) if limit is not None else L - 1)

    def _last_layer(self, nq, h, lay, B, L, pos, limit):
        """K/V for every row, Q / attention / O / MLP for each request's scored row only."""
        cfg = self.cfg
        qd, kd = cfg.q_dim, cfg.kv_dim
        dev = h.device
        kv = self._qkv_cols(lay, nq, qd, qd + 2 * kd)
        torch.ops.mica.qk_norm_rope(kv, None, lay.k_norm, self.cos, self.sin, pos, 0, 0, cfg.kv_heads, cfg.eps)
        k, v = kv.split([kd, kd], dim=1)
        rows = self._scored_rows(B, L, limit, dev)
        res = h.index_select(0, rows)
        qpos = (limit.view(B) - 1) if limit is not None else torch.full((B,), L - 1, dtype=torch.long, device=dev)
        mask = None
        if limit is not None:
            keys = torch.arange(L, device=dev)
            mask = torch.where(keys[None, :] < limit.view(B, 1), 0.0, float('-inf')).to(torch.bfloat16)
            mask = mask.view(B, 1, 1, L)
        q = self._qkv_cols(lay, nq, 0, qd, rows)
        torch.ops.mica.qk_norm_rope(q, lay.q_norm, None, self.cos, self.sin, qpos, 0, cfg.heads, 0, cfg.eps)
        attn = self._attention(q.view(B, 1, cfg.heads, cfg.head_dim), k.view(B, L, cfg.kv_heads, cfg.head_dim),
                               v.view(B, L, cfg.kv_heads, cfg.head_dim), causal=False, mask=mask)
        qa, sa = torch.ops.mica.act_quant(attn, lay.o_inv, K._round_code())
        o = self._gemm(qa, sa, lay.o_w, lay.o_s, lay.o_b)
        nm, res = self._normed(o, lay.post_norm, res, lay.mlp_in_inv(), lay.distinct_mlp_invs())
        d = self._mlp(nm, lay)
        return res + d

    def probs(self, h_last: torch.Tensor, lo=None, hi=None):
        """Final norm + gathered lm_head GEMV + option softmax (one library call)."""
        return torch.ops.mica.option_logits(h_last.contiguous(), self.rows, self.m.final_norm, lo, hi, self.cfg.eps,
                                            N.NORM_WEIGHT)

    def eager_bucket(self, n: int) -> int:
        """Padded length for an eager run: a multiple of EAGER_BUCKET, so request shapes (and
        the attention library's per-shape plans) repeat across requests."""
        return min(-(-n // EAGER_BUCKET) * EAGER_BUCKET, max(n, self.max_len))

    @torch.no_grad()
    def score(self, ids, lo=None, hi=None, graphs: bool = True):
        """ids: 1-D int64 tensor on the device; lo/hi: the option slice (ints, default all
        rows). Uses a captured graph when the request's bucket has one, else runs eagerly on
        ids padded to a 256-token bucket (`limit` masks the padding). Returns (logits, probs)
        fp32 [1, n_rows]."""
        n = int(ids.shape[0])
        if graphs and self.bucket(n) in self.graphs:
            return self.replay(ids, lo, hi)
        dev = ids.device
        limit = None
        L = self.eager_bucket(n)
        if L != n:
            padded = torch.zeros(L, dtype=ids.dtype, device=dev)
            padded[:n].copy_(ids)
            ids = padded
            limit = torch.full((1,), n, dtype=torch.long, device=dev)
        lo_t = None if lo is None else torch.tensor([int(lo)], dtype=torch.int32, device=dev)
        hi_t = None if hi is None else torch.tensor([int(hi)], dtype=torch.int32, device=dev)
        if lo_t is not None and hi_t is None:
            hi_t = torch.tensor([self.rows.shape[0]], dtype=torch.int32, device=dev)
        if hi_t is not None and lo_t is None:
            lo_t = torch.zeros(1, dtype=torch.int32, device=dev)
        return self.probs(self.hidden_last(ids, limit), lo_t, hi_t)

    @torch.no_grad()
    def score_batch(self, ids_list, slices=None, graphs: bool = True):
        """Scores several requests in one pass: ids padded to [B, L] (L a multiple of 64),
        each request's own length as its limit, per-request option slices (lo, hi).
        Returns (logits, probs) fp32 [B, n_rows]. Used for batches of similar lengths, like
        the reference's shaped batching (v0.5/serving/lib/release_runtime.py:1156-1227); a
        [B, L] shape with a captured graph (capture_batch) replays it, like the reference's
        batch graphs (release_runtime.py:644-647). The per-request lengths and slices travel
        in one pinned copy, so nothing here waits for the device."""
        dev = self.m.device
        B = len(ids_list)
        lens = [int(t.shape[0]) for t in ids_list]
        L = self.bucket(max(lens))
        rows = self.rows.shape[0]
        sl = slices if slices is not None else [(0, rows)] * B
        meta = torch.tensor(lens + [int(a) for a, _ in sl] + [int(b) for _, b in sl], dtype=torch.long)
        meta = meta.pin_memory().to(dev, non_blocking=True)
        e = self.batch_graphs.get((B, L)) if graphs else None
        if e is None:
            ids = torch.zeros(B, L, dtype=torch.long, device=dev)
            limit = meta[:B]
            lo, hi = (None, None) if slices is None else (meta[B:2 * B].int(), meta[2 * B:].int())
        else:
            ids, limit, lo, hi = e['ids'], e['limit'], e['lo'], e['hi']
            ids.zero_()
            limit.copy_(meta[:B])
            lo.copy_(meta[B:2 * B])
            hi.copy_(meta[2 * B:])
        for i, t in enumerate(ids_list):
            ids[i, :lens[i]].copy_(t)
        if e is None:
            return self.probs(self.hidden_last(ids, limit), lo, hi)
        e['graph'].replay()
        return e['out'][0].clone(), e['out'][1].clone()

    @torch.no_grad()
    def capture_batch(self, B: int, L: int):
        """Captures the prefill of a padded [B, L] batch (L a multiple of 64) with static ids,
        per-request limits and option slices; score_batch replays it for that shape. The
        reference's capture_batch (v0.5/serving/lib/release_runtime.py:670-689) keys its batch
        graphs the same way."""
        if L % BUCKET or L > self.max_len or B < 1:
            raise ValueError(f'batch shape {B} x {L}: L must be a multiple of {BUCKET} within {self.max_len}')
        dev = self.m.device
        ids = torch.zeros(B, L, dtype=torch.long, device=dev)
        limit = torch.full((B,), L, dtype=torch.long, device=dev)
        lo = torch.zeros(B, dtype=torch.int32, device=dev)
        hi = torch.full((B,), self.rows.shape[0], dtype=torch.int32, device=dev)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.probs(self.hidden_last(ids, limit), lo, hi)
        torch.cuda.current_stream(dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        if self.pool is None:
            self.pool = torch.cuda.graph_pool_handle()
        with torch.cuda.graph(g, pool=self.pool):
            out = self.probs(self.hidden_last(ids, limit), lo, hi)
        self.batch_graphs[B, L] = {'graph': g, 'ids': ids, 'limit': limit, 'lo': lo, 'hi': hi, 'out': out}
        return g

    # ---- CUDA graphs ------------------------------------------------------------------------
    def bucket(self, n: int) -> int:
        return -(-n // BUCKET) * BUCKET

    @torch.no_grad()
    def capture(self, length: int):
        """Captures the prefill of a `length`-token bucket (a multiple of 64)."""
        if length % BUCKET or length > self.max_len:
            raise ValueError(f'bucket {length} is not a multiple of {BUCKET} within {self.max_len}')
        dev = self.m.device
        ids = torch.zeros(length, dtype=torch.long, device=dev)
        limit = torch.full((1,), length, dtype=torch.long, device=dev)
        lo = torch.zeros(1, dtype=torch.int32, device=dev)
        hi = torch.full((1,), self.rows.shape[0], dtype=torch.int32, device=dev)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.probs(self.hidden_last(ids, limit), lo, hi)
        torch.cuda.current_stream(dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        if self.pool is None:
            self.pool = torch.cuda.graph_pool_handle()     # all buckets share one pool, as in the reference
        with torch.cuda.graph(g, pool=self.pool):
            out = self.probs(self.hidden_last(ids, limit), lo, hi)
        self.graphs[length] = {'graph': g, 'ids': ids, 'limit': limit, 'lo': lo, 'hi': hi, 'out': out}
        return g

    @torch.no_grad()
    def replay(self, ids, lo=None, hi=None):
        n = int(ids.shape[0])
        L = self.bucket(n)
        e = self.graphs[L]
        e['ids'][:n].copy_(ids)
        if n < L:
            e['ids'][n:].zero_()
        e['limit'].fill_(n)
        e['lo'].fill_(0 if lo is None else int(lo))
        e['hi'].fill_(self.rows.shape[0] if hi is None else int(hi))
        e['graph'].replay()
        return e['out']

    def release(self):
        self.graphs.clear()
        self.batch_graphs.clear()
        self.pool = None
