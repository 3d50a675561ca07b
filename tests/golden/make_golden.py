"""Generates tests/golden/*.npz by running the REFERENCE's own code on seeded inputs.

Run in the build container, where the reference checkout is available (it is read, never
copied; only inputs/outputs are saved):

    python tests/golden/make_golden.py /path/to/reference [set names, e.g. model_int8]

(or set MICA_REFERENCE to the reference checkout and name only the sets). The set
`model_full` (the BASELINE-scale decoder of full_model.py scored at 2048 and 32768 tokens,
about half an hour of CPU) and `model_full_band` (the same with fp32 attention, the reference's
own sensitivity to attention rounding) and `model_layer0` (layer 0's intermediates at full dims)
are made only when named.

What runs (all on CPU):
  * the reference's Triton kernels v0.5/serving/kernel_src/kernels.py act_quant and mm_i8,
    and lib/fused_kernels.py norm / swiglu, under Triton's CPU interpreter
    (TRITON_INTERPRET=1). The interpreter's fp32 -> bf16 cast truncates, so the Triton
    kernels write fp32 outputs here and the cast is applied afterwards (RNE, as on GPU);
  * the reference's torch path: int8_quant.quant_act / quant_weight / int_gemm_exact,
    int8_runtime.QLinear(..., backend='emulate'), fused_kernels.rms_norm / swi_glu CPU
    branches, and the readout of release_runtime.py:302-306 restated on a
    Qwen3RMSNorm + gathered lm_head rows.
"""
from __future__ import annotations

import os
import sys
import types
from pathlib import Path

os.environ['TRITON_INTERPRET'] = '1'

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
ARGS = sys.argv[1:]
if ARGS and Path(ARGS[0]).is_dir():
    REF = Path(ARGS.pop(0))
elif os.environ.get('MICA_REFERENCE'):
    REF = Path(os.environ['MICA_REFERENCE'])
else:
    sys.exit('usage: make_golden.py /path/to/reference [sets...]  (or set MICA_REFERENCE)')
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(REF / 'v0.5' / 'serving' / 'lib'))
sys.path.insert(0, str(REF / 'v0.5' / 'serving' / 'kernel_src'))

import fused_kernels as fk  # noqa: E402
import int8_quant as wq  # noqa: E402
import int8_runtime as rt  # noqa: E402
import kernels as ksrc  # noqa: E402

torch.set_num_threads(8)


def bits(t: torch.Tensor) -> np.ndarray:
    assert t.dtype == torch.bfloat16
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def triton_act_quant(x, inv):
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8)
    s = torch.empty((m,), dtype=torch.float32)
    ksrc.act_quant[(m,)](x, inv if inv is not None else s, q, s, k, x.stride(0), q.stride(0),
                         HAS_INV=inv is not None, BLOCK=1024)
    return q, s


def triton_mm_i8_f32(qx, qw, sx, sw, bias):
    m, k = qx.shape
    n = qw.shape[0]
    c = torch.empty((m, n), dtype=torch.float32)
    bm, bn = 16, 64
    grid = ((m + bm - 1) // bm) * ((n + bn - 1) // bn)
    ksrc.mm_i8[(grid,)](qx, qw, sx, sw, bias if bias is not None else sw, c, m, n, k, qx.stride(0), 1, qw.stride(0), 1,
                        c.stride(0), 1, HAS_BIAS=bias is not None, BM=bm, BN=bn, BK=128, GROUP_M=8)
    return c


def act_cases(g):
    out = {}
    for name, (m, k, smooth, outl) in {
        'a': (3, 2560, False, False),
        'b': (17, 4096, True, False),
        'c': (48, 2560, False, True),
        'd': (5, 9728, True, True),
        'e': (2, 64, False, False),
        'f': (4, 256, False, False),
    }.items():
        x = torch.randn(m, k, generator=g)
        if outl:
            ch = torch.randperm(k, generator=g)[:8]
            x[:, ch] *= 50
        x = x.to(torch.bfloat16)
        inv = (torch.rand(k, generator=g) * 2 + 0.1).float() if smooth else None
        if name == 'f':
            # tie-rich: absmax 127/8 gives scale exactly 1/8, so x = n/16 quantises to n/2
            x = (torch.round(torch.randn(m, k, generator=g) * 8) / 16).to(torch.bfloat16)
            x[:, 0] = 127 / 8
        q_away, s_away = triton_act_quant(x, inv)
        q_even, s_even = wq.quant_act(x, inv, 'int8')
        out[name] = dict(x=bits(x), inv=np.zeros(0, np.float32) if inv is None else inv.numpy(),
                         q_away=q_away.numpy(), s_away=s_away.numpy(), q_even=q_even.numpy(), s_even=s_even.numpy())
    return out


def gemm_cases(g):
    out = {}
    for name, (m, n, k, has_bias) in {
        'a': (7, 64, 2560, False),
        'b': (33, 32, 4096, True),
        'c': (130, 48, 512, False),
        'd': (1, 32, 9728, True),
    }.items():
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        w = (torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16)
        bias = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16) if has_bias else None
        lin = types.SimpleNamespace(weight=w, bias=bias)
        ql = rt.QLinear(lin, None, 'emulate')
        y_ref = ql(x)                                   # the reference's own QLinear (torch path)
        qx, sx = wq.quant_act(x, None, 'int8')
        acc = wq.int_gemm_exact(qx, ql.qweight)
        acc2 = wq.torch_int_mm(qx, ql.qweight)
        assert torch.equal(acc, acc2)
        y32 = triton_mm_i8_f32(qx, ql.qweight, sx, ql.wscale, ql.bias)  # the reference Triton kernel
        out[name] = dict(x=bits(x), bias=np.zeros(0, np.float32) if bias is None else ql.bias.numpy(),
                         qw=ql.qweight.numpy(), sw=ql.wscale.numpy(), qx=qx.numpy(), sx=sx.numpy(), acc=acc.numpy(),
                         y_triton_f32=y32.numpy(), y_qlinear=bits(y_ref))
    return out


@torch.no_grad()
def norm_cases(g):
    _, norm_k, swiglu_k = fk._kernels()
    out = {}
    for name, (m, k, with_res) in {'a': (4, 2560, False), 'b': (9, 2560, True), 'c': (3, 1024, True)}.items():
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        r = torch.randn(m, k, generator=g).to(torch.bfloat16) if with_res else None
        w = (torch.randn(k, generator=g) * 0.1).to(torch.bfloat16)   # (1 + w) convention
        eps = 1e-6
        res = fk.rms_norm(x, w, eps, r)                       # reference CPU branch
        y_cpu, s_cpu = (res if r is not None else (res, x))
        # reference Triton kernel, fp32 outputs
        y32 = torch.empty((m, k), dtype=torch.float32)
        s32 = torch.empty((m, k), dtype=torch.float32)
        xin = x
        norm_k[(m,)](xin, y32, w, r if r is not None else xin, s32, k, xin.stride(0),
                     (r if r is not None else xin).stride(0), eps, r is not None, 1 << (k - 1).bit_length())
        # HF Qwen3RMSNorm with a gamma ~ N(1, 0.1) weight
        from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm
        hf = Qwen3RMSNorm(k, eps=eps)
        gam = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
        hf.weight.data = gam.clone()
        hf = hf.to(torch.bfloat16)
        src = s_cpu if r is not None else x
        y_hf = hf(src)
        out[name] = dict(x=bits(x), r=np.zeros(0, np.uint16) if r is None else bits(r), w=bits(w), eps=np.float32(eps),
                         y_cpu=bits(y_cpu), sum_cpu=bits(s_cpu), y_triton_f32=y32.numpy(), gamma=bits(gam),
                         y_hf=bits(y_hf))
    # swiglu
    gt = (torch.randn(6, 1024, generator=g) * 3).to(torch.bfloat16)
    ut = torch.randn(6, 1024, generator=g).to(torch.bfloat16)
    y_cpu = fk.swi_glu(gt, ut)
    y32 = torch.empty((6, 1024), dtype=torch.float32)
    swiglu_k[(6,)](gt, ut, y32, gt.numel())
    out['swiglu'] = dict(g=bits(gt), u=bits(ut), y_cpu=bits(y_cpu), y_triton_f32=y32.numpy())
    return out


@torch.no_grad()
def readout_cases(g):
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm
    d, vocab, b = 256, 1000, 3
    lm = (torch.randn(vocab, d, generator=g) * 0.05).to(torch.bfloat16)
    ids = torch.randperm(vocab, generator=g)[:40]
    weight = lm.index_select(0, ids).float().clone()      # release_runtime.py:302
    norm = Qwen3RMSNorm(d, eps=1e-6)
    norm.weight.data = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    norm = norm.to(torch.bfloat16)
    h = torch.randn(b, d, generator=g).to(torch.bfloat16)
    hn = norm(h)
    z = torch.nn.functional.linear(hn.float(), weight).float()   # release_runtime.py:304-306
    lo = np.array([0, 2, 2], np.int32)
    hi = np.array([2, 40, 9], np.int32)
    probs = np.zeros((b, weight.shape[0]), np.float32)
    for i in range(b):
        probs[i, lo[i]:hi[i]] = z[i, lo[i]:hi[i]].softmax(-1).numpy()   # release_runtime.py:509-522
    return {'a': dict(h=bits(h), gamma=bits(norm.weight.data), rows=weight.numpy(), hn=bits(hn), logits=z.numpy(),
                      lo=lo, hi=hi, probs=probs)}


@torch.no_grad()
def selftest_cases(g):
    """Inputs shaped like the reference's start-up self-test (int8_runtime.py:362-443)."""
    gs = torch.Generator().manual_seed(rt.SELFTEST_SEED)
    n, k = 32, 2560
    w = (torch.randn(n, k, generator=gs) * 0.05).to(torch.bfloat16)
    amax = torch.rand(k, generator=gs) * 4 + 0.05
    amax[::61] *= 25.0
    smooth = wq.smooth_factors(amax, w, rt.ALPHA)
    lin = types.SimpleNamespace(weight=w, bias=None)
    q = rt.QLinear(lin, smooth, 'emulate')
    x = (torch.randn(24, k, generator=gs) * amax / 3).to(torch.bfloat16)
    y = q(x)
    return {'a': dict(amax=amax.numpy(), smooth=smooth.numpy(), inv=q.inv_smooth.numpy(),
                      qw=q.qweight.numpy(), sw=q.wscale.numpy(), x=bits(x), y=bits(y))}


MODEL_DIMS = dict(hidden_size=128, intermediate_size=256, num_hidden_layers=3, num_attention_heads=2,
                  num_key_value_heads=1, head_dim=64, vocab_size=512, rms_norm_eps=1e-6, rope_theta=1e6,
                  tie_word_embeddings=True)


@torch.no_grad()
def model_cases(g):
    """A tiny dense Qwen3 decoder scored the reference way: every projection converted by
    the reference's int8_runtime.convert (QLinear 'emulate': quant_act half-even + exact int
    GEMM + dequant), last hidden state of the final norm, fp32 linear over gathered label
    rows (release_runtime.py:302-306), softmax over the option slice (:509-522)."""
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(**MODEL_DIMS)
    cfg._attn_implementation = 'eager'
    torch.manual_seed(20261202)
    model = Qwen3ForCausalLM(cfg).eval()
    for name, prm in model.named_parameters():
        if name.endswith('norm.weight'):
            prm.data = 1 + 0.1 * torch.randn(prm.shape, generator=g)
    model = model.to(torch.bfloat16)
    state = {k: v.clone() for k, v in model.state_dict().items()}
    replaced, _ = rt.convert(model.model, None, 'emulate')
    assert replaced == 7 * cfg.num_hidden_layers
    options = torch.randperm(cfg.vocab_size, generator=g)[:40]
    weight = model.get_output_embeddings().weight.detach().index_select(0, options).float().clone()
    out = {'state/' + k: bits(v) for k, v in state.items() if v.dtype == torch.bfloat16}
    out['options'] = options.numpy().astype(np.int64)
    for i, n in enumerate((37, 100)):
        ids = torch.randint(0, cfg.vocab_size, (n,), generator=g)
        hid = model.model(ids[None]).last_hidden_state[:, -1]
        z = torch.nn.functional.linear(hid.float(), weight).float()
        lo, hi = (2, 2 + 17) if i == 0 else (0, 40)
        p = torch.zeros_like(z)
        p[:, lo:hi] = z[:, lo:hi].softmax(-1)
        out[f'ids{i}'] = ids.numpy().astype(np.int64)
        out[f'hidden{i}'] = bits(hid)
        out[f'logits{i}'] = z.numpy()
        out[f'probs{i}'] = p.numpy()
        out[f'slice{i}'] = np.array([lo, hi], np.int32)
    return {'m': out}


@torch.no_grad()
def model_int8_cases(g):
    """An int8-w8a8/1 weights folder (model_int8/: model-int8.safetensors + config.json) of a
    tiny dense Qwen3 converted by the reference's int8_runtime.convert WITH activation
    statistics, so its QLinears carry inv_smooth (lib/int8_runtime.py:195-206):
      layer 0: no statistics (no smoothing: the fused q|k|v and gate|up paths);
      layer 1: statistics for every projection (per-projection smoothing: q, k, v and gate,
               up each quantise their shared input differently);
      layer 2: statistics for o_proj and down_proj only (the fused MLP with down smoothing).
    The file holds the converted model's state dict (the reference QLinear buffer names), with
    lm_head tied to the embedding through the `ties` metadata; golden option probabilities come
    from the converted model itself (QLinear 'emulate')."""
    import json
    from safetensors.torch import save_file
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(**MODEL_DIMS)
    cfg._attn_implementation = 'eager'
    torch.manual_seed(20261203)
    model = Qwen3ForCausalLM(cfg).eval()
    for name, prm in model.named_parameters():
        if name.endswith('norm.weight'):
            prm.data = 1 + 0.1 * torch.randn(prm.shape, generator=g)
    model = model.to(torch.bfloat16)

    def amax(k):
        a = torch.exp(torch.randn(k, generator=g))
        a[torch.randperm(k, generator=g)[:4]] *= 20.0          # outlier channels
        return a

    H, Q, I = cfg.hidden_size, cfg.num_attention_heads * cfg.head_dim, cfg.intermediate_size
    stats = {}
    x_attn, x_mlp = amax(H), amax(H)
    for n in ('q_proj', 'k_proj', 'v_proj'):
        stats[f'layers.1.self_attn.{n}'] = x_attn                 # one input, per-projection factors
    for n in ('gate_proj', 'up_proj'):
        stats[f'layers.1.mlp.{n}'] = x_mlp
    for i in (1, 2):
        stats[f'layers.{i}.self_attn.o_proj'] = amax(Q)
        stats[f'layers.{i}.mlp.down_proj'] = amax(I)
    replaced, smoothed = rt.convert(model.model, stats, 'emulate')
    assert replaced == 7 * cfg.num_hidden_layers and smoothed == 9, (replaced, smoothed)
    state = model.state_dict()
    ties = {'lm_head.weight': 'model.embed_tokens.weight'}
    stored = {k: v.contiguous() for k, v in state.items() if k not in ties}
    folder = HERE / 'model_int8'
    folder.mkdir(exist_ok=True)
    save_file(stored, str(folder / rt.FILE), metadata={'format': rt.FILE_FORMAT, 'ties': json.dumps(ties)})
    (folder / 'config.json').write_text(json.dumps({**MODEL_DIMS, 'architectures': ['Qwen3ForCausalLM'],
                                                    'model_type': 'qwen3'}, indent=1, sort_keys=True) + '\n')
    options = torch.randperm(cfg.vocab_size, generator=g)[:40]
    weight = model.get_output_embeddings().weight.detach().index_select(0, options).float().clone()
    out = {'options': options.numpy().astype(np.int64)}
    for i, n in enumerate((45, 130)):
        ids = torch.randint(0, cfg.vocab_size, (n,), generator=g)
        hid = model.model(ids[None]).last_hidden_state[:, -1]
        z = torch.nn.functional.linear(hid.float(), weight).float()
        lo, hi = (2, 2 + 23) if i == 0 else (0, 40)
        p = torch.zeros_like(z)
        p[:, lo:hi] = z[:, lo:hi].softmax(-1)
        out[f'ids{i}'] = ids.numpy().astype(np.int64)
        out[f'logits{i}'] = z.numpy()
        out[f'probs{i}'] = p.numpy()
        out[f'slice{i}'] = np.array([lo, hi], np.int32)
    return {'m': out}


def _register_fp32_attention():
    """'sdpa_fp32': HF's SDPA attention with q, k, v upcast to fp32 and the output cast back,
    a more accurate attention than the served bf16 one, used to measure how far the reference
    model's own probabilities move under an attention rounding change."""
    from transformers import AttentionInterface
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    def fp32_forward(module, query, key, value, attention_mask, **kwargs):
        out, w = sdpa_attention_forward(module, query.float(), key.float(), value.float(), attention_mask, **kwargs)
        return out.to(query.dtype), w

    AttentionInterface.register('sdpa_fp32', fp32_forward)


@torch.no_grad()
def model_full_cases(layers=None, lengths=None, attn='sdpa'):
    """The BASELINE-scale decoder of full_model.py (4B dims, 36 layers, vocab 151936) scored
    the reference way: HF Qwen3ForCausalLM (bf16, SDPA attention) with every projection
    converted by the reference's int8_runtime.convert (QLinear 'emulate': quant_act
    half-even + exact int GEMM + dequant, lib/int8_runtime.py:172-206), the final norm's
    last row, an fp32 linear over the 257 gathered rows (release_runtime.py:302-306) and
    the softmax over the 255 options (:509-522). Only ids, rows, hidden state, logits and
    probabilities are saved; the weights are regenerated from full_model.SEED."""
    import time
    import full_model as FM
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding
    dims = dict(FM.HF_CONFIG)
    if layers is not None:
        dims['num_hidden_layers'] = layers
    cfg = Qwen3Config(**dims)
    if attn == 'sdpa_fp32':
        _register_fp32_attention()
    cfg._attn_implementation = attn
    with torch.device('meta'):
        model = Qwen3ForCausalLM(cfg)
    model.load_state_dict(FM.state(cfg.num_hidden_layers), assign=True)
    model.model.rotary_emb = Qwen3RotaryEmbedding(cfg)      # fp32 inv_freq, built off the meta device
    model.eval()
    bad = [n for n, t in list(model.named_parameters()) + list(model.named_buffers()) if t.is_meta]
    assert not bad, bad
    replaced, _ = rt.convert(model.model, None, 'emulate')
    assert replaced == 7 * cfg.num_hidden_layers
    out = {}
    for n in (lengths or FM.LENGTHS):
        ids, rows = FM.request(n)
        t0 = time.time()
        hid = model.model(ids[None]).last_hidden_state[:, -1]
        weight = model.lm_head.weight.detach().index_select(0, rows).float()
        z = torch.nn.functional.linear(hid.float(), weight).float()
        lo, hi = FM.OPTION_SLICE
        p = torch.zeros_like(z)
        p[:, lo:hi] = z[:, lo:hi].softmax(-1)
        print(f'model_full ({attn}): {n} tokens in {time.time() - t0:.0f} s', flush=True)
        out[f'n{n}'] = dict(ids=ids.numpy().astype(np.int32), rows=rows.numpy().astype(np.int32), hidden=bits(hid),
                            logits=z.numpy(), probs=p.numpy(), slice=np.array([lo, hi], np.int32))
    return out


@torch.no_grad()
def model_layer0_cases():
    """Layer 0 of the BASELINE-scale decoder of full_model.py on the 2048-token request, as the
    reference computes it (HF Qwen3 decoder layer, every projection a QLinear 'emulate',
    SDPA attention): for the last 4 rows, the attention output that o_proj quantises, o_proj's
    output, the post-attention norm, the SwiGLU product that down_proj quantises, down_proj's
    output and the layer's output. Given the same attention output, every later step of a
    layer is exact integer arithmetic plus single roundings, so a W8A8 layer can reproduce
    these bit for bit."""
    import full_model as FM
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding
    dims = dict(FM.HF_CONFIG)
    dims['num_hidden_layers'] = 1
    cfg = Qwen3Config(**dims)
    cfg._attn_implementation = 'sdpa'
    with torch.device('meta'):
        model = Qwen3ForCausalLM(cfg)
    model.load_state_dict(FM.state(1), assign=True)
    model.model.rotary_emb = Qwen3RotaryEmbedding(cfg)
    model.eval()
    rt.convert(model.model, None, 'emulate')
    lay = model.model.layers[0]
    cap = {}

    def out_hook(name):
        def hook(mod, inp, out):
            cap[name] = (out[0] if isinstance(out, tuple) else out)[0, -4:].contiguous()
        return hook

    def in_hook(name):
        def hook(mod, inp):
            cap[name] = inp[0][0, -4:].contiguous()
        return hook

    lay.self_attn.o_proj.register_forward_pre_hook(in_hook('attn'))
    lay.self_attn.o_proj.register_forward_hook(out_hook('o_proj'))
    lay.post_attention_layernorm.register_forward_hook(out_hook('ln2'))
    lay.mlp.down_proj.register_forward_pre_hook(in_hook('h'))
    lay.mlp.down_proj.register_forward_hook(out_hook('down'))
    lay.register_forward_hook(out_hook('layer_out'))
    ids, _ = FM.request(2048)
    model.model(ids[None])
    return {'l0': {k: bits(v) for k, v in cap.items()}}


def save(name, cases):
    flat = {f'{c}/{k}': v for c, d in cases.items() for k, v in d.items()}
    np.savez_compressed(HERE / f'{name}.npz', **flat)
    print(name, sum(v.nbytes for v in flat.values()) // 1024, 'KiB raw')


if __name__ == '__main__':
    # optional names after the reference path regenerate only those sets
    only = set(ARGS)
    g = torch.Generator().manual_seed(20261201)
    for name, fn in (('act_quant', act_cases), ('gemm', gemm_cases), ('norm', norm_cases),
                     ('readout', readout_cases), ('selftest', selftest_cases), ('model', model_cases)):
        cases = fn(g)                     # every set draws from the one generator, in this order
        if not only or name in only:
            save(name, cases)
    if not only or 'model_int8' in only:
        save('model_int8', model_int8_cases(torch.Generator().manual_seed(20261203)))
    if 'model_full' in only:
        save('model_full', model_full_cases())
    if 'model_layer0' in only:
        save('model_layer0', model_layer0_cases())
    if 'model_full_band' in only:
        # the same model and requests with fp32 attention: the reference's own sensitivity
        save('model_full_band', model_full_cases(attn='sdpa_fp32'))
