"""The reference engine, unmodified, running on this repo's B200 kernels.

The reference's ``TransformerLM`` / ``Attention.forward`` / ``generate`` /
``speculative_generate`` / ``InferenceEngine`` are imported from its installed
copy (``tests/refengine.py`` composes it behind this repo's ``engine`` and
``kernels`` packages), so every attention call, paged append, gather and INT8
projection they make lands in ``libcie_attn.so`` through their own imports.

The properties are the reference's own tests, restated here because its test
files are not installed with it:

* tests/model/test_transformer_forward.py:6-46 — logits shape and cache growth,
  determinism, token-by-token decoding matches one prefill (atol 1e-3);
* tests/decode/test_speculative.py:25-37 — greedy speculative decoding with
  draft == target reproduces the base loop;
* tests/kernels/test_triton_kernels.py:11-42 — the attention and INT8 kernels
  against ``kernels.ref`` (max abs 1e-3, fp16).

Each engine property runs in two modes: ``unchanged`` (the reference's
Attention.forward as it ships: its own RoPE, append, gather, then
``engine.attention.flash_attention``) and ``fused`` (the same modules rerouted
through ``engine.attention.use_fused_attention``: RoPE fused into the paged
append and the attention kernels, paged decode). fp16 is the engine's dtype
policy (engine/dtype.py:8-11); bf16 runs the same model cast to bf16.
Beyond the reference's tiny model, a Llama-like geometry (GQA 4, d = 64 / 128,
300-token prompts, chunked prefill, decode) is checked against the same model
whose attention is the reference's fp32 ``flash_attention_ref``.
"""

from __future__ import annotations

import math

import pytest

from tests.refengine import compose, origin, reference_root

ROOT = reference_root()
needs_ref = pytest.mark.skipif(
    ROOT is None, reason="reference engine not installed (baseline/_ref or $CIE_REFERENCE_ENGINE)")

MODES = ["unchanged", "fused"]
DTYPES = ["fp16", "bf16"]


@pytest.fixture(scope="module")
def ref():
    """The composed namespace: reference modules with this repo's kernels underneath."""
    compose(ROOT)
    import types

    import engine.attention as attention
    import engine.cache.kv_cache as kv_cache
    import engine.config as config
    import engine.decode.base_loop as base_loop
    import engine.decode.speculative as speculative
    import engine.dtype as dtype
    import engine.model as model
    import engine.model.block as block
    import engine.model.loader as loader
    import engine.model.norm as norm
    import engine.quant as quant
    import engine.runtime as runtime
    import engine.tokenizer as tokenizer
    import kernels.ref as kref

    return types.SimpleNamespace(
        attention=attention, kv_cache=kv_cache, config=config, base_loop=base_loop,
        speculative=speculative, dtype=dtype, model=model, block=block, loader=loader,
        norm=norm, quant=quant, runtime=runtime, tokenizer=tokenizer, kref=kref)


# ---------------------------------------------------------------- CPU: composition
@needs_ref
def test_reference_modules_compose_over_this_repo(ref):
    import engine.attention
    import engine.cache.block_table
    import kernels.flash_attention
    import kernels.int8_matmul

    for m in (engine.attention, engine.cache.kv_cache, engine.cache.block_table,
              kernels.flash_attention, kernels.int8_matmul):
        assert origin(m) == "repo", m.__name__
    for m in (ref.block, ref.model, ref.base_loop, ref.speculative, ref.runtime, ref.kref,
              ref.quant, ref.config):
        assert origin(m) == "reference", m.__name__
    # the reference's block imports the call site and the cache from this repo
    assert ref.block.flash_attention is engine.attention.flash_attention
    assert ref.block.PagedKVCache is ref.kv_cache.PagedKVCache
    assert ref.block.PagedKVCache.__module__ == "engine.cache.kv_cache"


# ---------------------------------------------------------------- helpers
def _torch_dtype(name):
    import torch

    return {"fp16": torch.float16, "bf16": torch.bfloat16}[name]


def _tiny_cfg(ref, **overrides):
    """The reference's tests/conftest.py:28-43 model geometry."""
    cfg = ref.config.ModelConfig(vocab_size=32, hidden_size=32, num_layers=2, num_heads=2,
                                 num_kv_heads=2, head_dim=16, max_position_embeddings=64,
                                 intermediate_size=64)
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg


def _make_cache(ref, cfg, device, dtype, num_blocks=32, block_size=8):
    """tests/conftest.py:46-56 of the reference (num_blocks 32, block size 8)."""
    kc = ref.kv_cache
    return kc.PagedKVCache(kc.KVCacheConfig(num_layers=cfg.num_layers,
                                            num_kv_heads=cfg.num_kv_heads,
                                            head_dim=cfg.head_dim, num_blocks=num_blocks,
                                            block_size=block_size, dtype=dtype, device=device))


def _prepare(ref, model, device, dtype, mode):
    model = model.to(device)
    ref.runtime.cast_non_quantized_params(model, dtype)
    if mode == "fused":
        n = ref.attention.use_fused_attention(model)
        assert n == model.cfg.num_layers
    return model


def _tiny_model(ref, cfg, device, dtype, mode, seed=0):
    """tests/conftest.py:59-63 of the reference, in the given dtype and mode."""
    m = ref.loader.randomize_weights(ref.model.build_target(cfg), seed=seed)
    return _prepare(ref, m, device, dtype, mode)


def _kv_dtype(ref, device, name):
    # fp16: the engine's own policy (engine/dtype.py:14-16); bf16: relaxed here
    return ref.dtype.kv_cache_dtype(device) if name == "fp16" else _torch_dtype(name)


def _act_dtype(ref, device, name):
    return ref.dtype.activation_dtype(device) if name == "fp16" else _torch_dtype(name)


# ---------------------------------------------------------------- GPU: the reference's tests
@needs_ref
@pytest.mark.gpu
@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("mode", MODES)
def test_forward_shape_and_cache_growth(ref, cuda, mode, dt):
    import torch

    cfg = _tiny_cfg(ref)
    model = _tiny_model(ref, cfg, cuda, _act_dtype(ref, cuda, dt), mode)
    cache = _make_cache(ref, cfg, cuda, _kv_dtype(ref, cuda, dt))
    table = cache.new_sequence()
    logits = model(torch.tensor([[1, 2, 3, 4, 5]], device=cuda), cache, table)
    assert logits.shape == (1, 5, cfg.vocab_size)
    assert table.length == 5
    assert torch.isfinite(logits.float()).all()


@needs_ref
@pytest.mark.gpu
@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("mode", MODES)
def test_forward_is_deterministic(ref, cuda, mode, dt):
    import torch

    cfg = _tiny_cfg(ref)
    model = _tiny_model(ref, cfg, cuda, _act_dtype(ref, cuda, dt), mode, seed=42)
    tokens = torch.tensor([[7, 3, 1]], device=cuda)
    outs = []
    for _ in range(2):
        cache = _make_cache(ref, cfg, cuda, _kv_dtype(ref, cuda, dt))
        outs.append(model(tokens, cache, cache.new_sequence()))
    assert torch.equal(outs[0], outs[1])


@needs_ref
@pytest.mark.gpu
@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("mode", MODES)
def test_incremental_forward_matches_full(ref, cuda, mode, dt):
    """3 tokens at once vs one by one: last-step logits agree within 1e-3."""
    import torch

    cfg = _tiny_cfg(ref)
    model = _tiny_model(ref, cfg, cuda, _act_dtype(ref, cuda, dt), mode, seed=1)
    tokens = torch.tensor([[5, 2, 9]], device=cuda)
    cache_full = _make_cache(ref, cfg, cuda, _kv_dtype(ref, cuda, dt))
    full = model(tokens, cache_full, cache_full.new_sequence())
    cache_inc = _make_cache(ref, cfg, cuda, _kv_dtype(ref, cuda, dt))
    table_inc = cache_inc.new_sequence()
    for i in range(tokens.shape[1]):
        step = model(tokens[:, i:i + 1], cache_inc, table_inc)
    assert torch.allclose(step[0, -1].float(), full[0, -1].float(), atol=1e-3)


def _clone_models(ref, cfg, seed, device, dtype, mode):
    """tests/decode/test_speculative.py:11-22: two models with identical weights."""
    m1 = ref.loader.randomize_weights(ref.model.build_target(cfg), seed=seed)
    m2 = ref.model.build_target(cfg)
    m2.load_state_dict(m1.state_dict())
    return _prepare(ref, m1, device, dtype, mode), _prepare(ref, m2, device, dtype, mode)


@needs_ref
@pytest.mark.gpu
@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("mode", MODES)
def test_speculative_matches_base_loop_when_draft_equals_target(ref, cuda, mode, dt):
    cfg = _tiny_cfg(ref)
    act, kvd = _act_dtype(ref, cuda, dt), _kv_dtype(ref, cuda, dt)
    target, _ = _clone_models(ref, cfg, 3, cuda, act, mode)
    prompt = [1, 4, 2]
    base = list(ref.base_loop.generate(target, prompt, _make_cache(ref, cfg, cuda, kvd),
                                       max_new_tokens=8))
    target2, draft2 = _clone_models(ref, cfg, 3, cuda, act, mode)
    spec = list(ref.speculative.speculative_generate(
        target2, draft2, prompt, _make_cache(ref, cfg, cuda, kvd),
        _make_cache(ref, cfg, cuda, kvd), max_new_tokens=8, gamma=3))
    assert spec == base


@needs_ref
@pytest.mark.gpu
def test_flash_attention_matches_reference_kernel_test(ref, cuda):
    """tests/kernels/test_triton_kernels.py:11-22 against this repo's entry point."""
    import torch

    from kernels.flash_attention import flash_attention

    torch.manual_seed(0)
    B, H, Lq, Lk, D = 2, 4, 64, 64, 64
    q = torch.randn(B, H, Lq, D, device=cuda, dtype=torch.float16)
    k = torch.randn(B, H, Lk, D, device=cuda, dtype=torch.float16)
    v = torch.randn(B, H, Lk, D, device=cuda, dtype=torch.float16)
    out = flash_attention(q, k, v, causal=True)
    expect = ref.kref.flash_attention_ref(q, k, v, causal=True)
    assert (out - expect).abs().max() < 1e-3


@needs_ref
@pytest.mark.gpu
def test_int8_matmul_matches_reference_kernel_test(ref, cuda):
    """tests/kernels/test_triton_kernels.py:25-42 against this repo's entry point."""
    import torch

    from kernels.int8_matmul import int8_matmul

    torch.manual_seed(0)
    M, N, K = 64, 128, 64
    w_fp = torch.randn(N, K)
    scales = (w_fp.abs().amax(dim=1) / 127.0).clamp_min(1e-8)
    w_int8 = (w_fp / scales.unsqueeze(-1)).round().clamp(-128, 127).to(torch.int8)
    x = torch.randn(M, K, dtype=torch.float16, device=cuda)
    y = int8_matmul(x, w_int8.to(cuda), scales.to(cuda, torch.float16))
    expect = ref.kref.int8_matmul_ref(x, w_int8.to(cuda), scales.to(cuda, torch.float16))
    assert (y - expect).abs().max() < 1e-3


# ---------------------------------------------------------------- GPU: engine.generate()
def _char_engine(ref, cuda, spec: bool, seed: int):
    cfg_kw = dict(hidden_size=128, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=32,
                  max_position_embeddings=256, intermediate_size=256)
    tok = ref.tokenizer.CharTokenizer()
    cfg = ref.config.ModelConfig(vocab_size=tok.vocab_size, **cfg_kw)
    target = _unit_scale(ref, ref.model.build_target(cfg), seed)
    draft = None
    spec_cfg = None
    if spec:
        dcfg = ref.config.ModelConfig(vocab_size=tok.vocab_size, **dict(cfg_kw, num_layers=1))
        draft = _unit_scale(ref, ref.model.build_draft(cfg, dcfg), seed + 1)
        draft = draft.to(cuda)
        ref.runtime.cast_non_quantized_params(draft, ref.dtype.activation_dtype(cuda))
        spec_cfg = ref.config.SpecConfig(gamma=3, enabled=True)
    eng_cfg = ref.config.EngineConfig(num_kv_blocks=128, kv_block_size=16)
    eng = ref.runtime.build_engine(cfg, eng_cfg, tok, target=target)
    eng.draft, eng.spec_cfg = draft, spec_cfg
    return eng


@needs_ref
@pytest.mark.gpu
def test_engine_generate_speculative_equals_base(ref, cuda):
    """InferenceEngine.generate (engine/runtime.py:72-103) end to end: greedy
    speculative decoding with an unrelated 1-layer draft must emit exactly the
    target's greedy tokens (the rejection rule keeps the target's choice), which
    exercises verify blocks (M = gamma + 1), rejections and cache rollback; a
    second call reuses the long-lived caches."""
    base = _char_engine(ref, cuda, spec=False, seed=11)
    spec = _char_engine(ref, cuda, spec=True, seed=11)
    for prompt in ("hello paged world", "the quick brown fox"):
        ids_b, ids_s = [], []
        text_b = base.generate(prompt, max_new_tokens=24).collect(lambda t, _: ids_b.append(t))
        text_s = spec.generate(prompt, max_new_tokens=24).collect(lambda t, _: ids_s.append(t))
        assert ids_s == ids_b and text_s == text_b
        assert len(ids_b) > 0


# ---------------------------------------------------------------- GPU: vs fp32 attention
def _unit_scale(ref, m, seed):
    """Weights at unit scale for the reference's modules (randomize_weights' +-0.02
    everywhere leaves fp16 activations and logits near zero, where near-ties
    abound): N(0, 1) embeddings, RMSNorm weights 1, int8 weights with scales
    that keep activations O(1)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        m.embed.weight.copy_(torch.randn(m.embed.weight.shape, generator=g))
        for mod in m.modules():
            if isinstance(mod, ref.norm.RMSNorm):
                mod.weight.fill_(1.0)
            if isinstance(mod, ref.quant.Int8Linear):
                mod.weight_int8.copy_(torch.randint(-127, 128, mod.weight_int8.shape, generator=g,
                                                    dtype=torch.int8))
                mod.scales.fill_(1.0 / (73.0 * math.sqrt(mod.in_features)))
    return m


def _llama_like(ref, d, seed):
    cfg = ref.config.ModelConfig(vocab_size=96, hidden_size=256, num_layers=2, num_heads=8,
                                 num_kv_heads=2, head_dim=d, max_position_embeddings=1024,
                                 intermediate_size=512, rope_theta=500000.0)
    return cfg, _unit_scale(ref, ref.model.build_target(cfg), seed)


def _run_schedule(model, cache, tokens, cuda):
    """300-token prompt (prefill), a 100-token chunk over that history (chunked
    prefill), then 6 single-token decode steps; returns the logits of each stage."""
    import torch

    t = cache.new_sequence()
    out = [model(tokens[:, :300], cache, t)[0, -1].float()]
    out.append(model(tokens[:, 300:400], cache, t)[0, -1].float())
    for i in range(400, 406):
        last = model(tokens[:, i:i + 1], cache, t)
    out.append(last[0, -1].float())
    assert t.length == 406
    return torch.stack(out)


@needs_ref
@pytest.mark.gpu
@pytest.mark.parametrize("d", [64, 128])
def test_engine_logits_match_fp32_attention(ref, cuda, monkeypatch, d):
    """Both modes against the same model whose attention is the reference's fp32
    flash_attention_ref (the oracle of the path): prefill on the tcgen05 kernel,
    chunked prefill, and decode (split-KV), fp16 as the engine runs."""
    import torch

    tokens = torch.randint(0, 96, (1, 406), generator=torch.Generator().manual_seed(d)).to(cuda)
    results = {}
    for mode in ("oracle", "unchanged", "fused"):
        cfg, m = _llama_like(ref, d, seed=d)
        model = _prepare(ref, m, cuda, torch.float16, "fused" if mode == "fused" else "unchanged")
        if mode == "oracle":
            def fa32(q, k, v, causal=False, scale=None):
                return ref.kref.flash_attention_ref(q, k, v, causal=causal, scale=scale)
            monkeypatch.setattr(ref.block, "flash_attention", fa32)
        cache = _make_cache(ref, cfg, cuda, torch.float16, num_blocks=64, block_size=16)
        with torch.no_grad():
            results[mode] = _run_schedule(model, cache, tokens, cuda)
        monkeypatch.undo()
    ora = results["oracle"]
    scale = ora.abs().mean(dim=-1, keepdim=True)
    for mode in ("unchanged", "fused"):
        err = (results[mode] - ora).abs()
        rel_max = (err.max(dim=-1).values / scale[:, 0]).max().item()
        rel_mean = (err.mean(dim=-1) / scale[:, 0]).max().item()
        # logits after two layers of fp16 activations: agree with the fp32-attention
        # model to within 5% of the mean logit magnitude at worst, 1% on average
        assert rel_max <= 5e-2 and rel_mean <= 1e-2, (mode, rel_max, rel_mean)
        print(f"d={d} {mode}: max err {rel_max:.2e}, mean err {rel_mean:.2e} "
              "(relative to the mean |logit|)")
