"""Engine-level GPU tests in the style of the reference's own:

* the paged cache on the GPU replays the reference's golden lifecycle (block ids,
  append, fork, rollback, free) with bit-exact gathers (tests/cache/test_kv_cache.py);
* attention_forward (fused RoPE + paged append + paged/prefill attention) on a
  tiny decoder: feeding tokens one by one matches one prefill
  (tests/model/test_transformer_forward.py:32-46), and greedy speculative
  decoding with draft == target reproduces the base loop
  (tests/decode/test_speculative.py:25-37), which exercises verify (M = gamma+1)
  and cache rollback.

The tiny decoder below is test scaffolding (embedding, one attention block per
layer through engine.attention.attention_forward, a SwiGLU-free MLP, LM head);
only the attention path is the product.
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from tests.helpers import assert_close_attn

pytestmark = pytest.mark.gpu


def test_cache_lifecycle_matches_reference(cuda, golden):
    import torch

    from engine.cache import KVCacheConfig, PagedKVCache

    log = json.loads(bytes(golden["life_log"]).decode())
    cache = PagedKVCache(KVCacheConfig(num_layers=2, num_kv_heads=2, head_dim=16, num_blocks=12,
                                       block_size=4, dtype=torch.bfloat16, device=cuda))
    rng = np.random.default_rng(1234)
    a, b = cache.new_sequence(), cache.new_sequence()

    def rows(n):
        return torch.from_numpy(rng.standard_normal((n, 2, 16)).astype(np.float32)).to(
            cuda, torch.bfloat16)

    mine, written = [], {"a": [[], []], "f": None}
    for layer in range(2):
        k, v = rows(6), rows(6)
        cache.append(layer, a, k, v, start=0)
        written["a"][layer].append((0, k, v))
    mine.append(["append_a6", list(a.blocks), a.length, list(cache._free)])
    for layer in range(2):
        cache.append(layer, b, rows(3), rows(3), start=0)
    mine.append(["append_b3", list(b.blocks), b.length, list(cache._free)])
    for layer in range(2):
        k, v = rows(3), rows(3)
        cache.append(layer, a, k, v, start=6)
        written["a"][layer].append((6, k, v))
    mine.append(["append_a3", list(a.blocks), a.length, list(cache._free)])
    f = cache.fork(a)
    fk0 = [cache.gather(layer, a)[0].clone() for layer in range(2)]
    mine.append(["fork_a", list(f.blocks), f.length, list(cache._free)])
    cache.rollback(a, 5)
    mine.append(["rollback_a5", list(a.blocks), a.length, list(cache._free)])
    for layer in range(2):
        k, v = rows(4), rows(4)
        cache.append(layer, a, k, v, start=5)
        written["a"][layer].append((5, k, v))
    mine.append(["append_a4", list(a.blocks), a.length, list(cache._free)])
    cache.free_sequence(b)
    mine.append(["free_b", list(b.blocks), b.length, list(cache._free)])
    assert mine == [list(x) for x in log]
    for layer in range(2):
        # expected contents: later writes overwrite earlier positions
        exp_k = torch.zeros(a.length, 2, 16, dtype=torch.bfloat16, device=cuda)
        for start, k, _ in written["a"][layer]:
            n = min(k.shape[0], a.length - start)
            exp_k[start:start + n] = k[:n]
        gk, _ = cache.gather(layer, a)
        assert torch.equal(gk, exp_k)
        # the fork kept its deep copy
        assert torch.equal(cache.gather(layer, f)[0], fk0[layer])


class TinyDecoder:
    """Embedding -> n x [attention (engine.attention_forward) + MLP] -> LM head."""

    def __init__(self, vocab, hidden, layers, hq, hkv, d, max_pos, device, seed=0):
        import torch

        from kernels import build_rope_cache

        g = torch.Generator().manual_seed(seed)
        r = lambda *s: (torch.rand(*s, generator=g) * 0.2 - 0.1).to(device, torch.bfloat16)  # noqa
        self.hq, self.hkv, self.d = hq, hkv, d
        self.emb = r(vocab, hidden)
        self.layers = [dict(wq=r(hidden, hq * d), wk=r(hidden, hkv * d), wv=r(hidden, hkv * d),
                            wo=r(hq * d, hidden), w1=r(hidden, 2 * hidden), w2=r(2 * hidden, hidden))
                       for _ in range(layers)]
        self.head = r(hidden, vocab)
        self.rope = build_rope_cache(max_pos, d, theta=10000.0, device=device)

    def forward(self, tokens, cache, table):
        import torch

        from engine.attention import attention_forward

        L = tokens.shape[0]
        start = table.length
        x = self.emb[tokens]  # (L, hidden)
        for i, p in enumerate(self.layers):
            q = (x @ p["wq"]).view(1, L, self.hq, self.d).transpose(1, 2)
            k = (x @ p["wk"]).view(1, L, self.hkv, self.d).transpose(1, 2)
            v = (x @ p["wv"]).view(1, L, self.hkv, self.d).transpose(1, 2)
            o = attention_forward(q, k, v, cache, i, table, start=start, rope=self.rope)
            x = x + o.transpose(1, 2).reshape(L, self.hq * self.d) @ p["wo"]
            x = x + torch.relu(x @ p["w1"]) @ p["w2"]
        return (x.float() @ self.head.float())  # (L, vocab)


def _cache(cfg_layers, hkv, d, device, blocks=64, bs=8):
    import torch

    from engine.cache import KVCacheConfig, PagedKVCache

    return PagedKVCache(KVCacheConfig(num_layers=cfg_layers, num_kv_heads=hkv, head_dim=d,
                                      num_blocks=blocks, block_size=bs, dtype=torch.bfloat16,
                                      device=device))


@pytest.mark.parametrize("geom", [(2, 2, 16), (8, 2, 64), (4, 1, 128)],
                         ids=["tiny_d16", "gqa4_d64", "gqa4_d128"])
def test_incremental_forward_matches_full(cuda, geom):
    import torch

    hq, hkv, d = geom
    model = TinyDecoder(32, 32, 2, hq, hkv, d, 256, cuda, seed=1)
    tokens = torch.tensor([5, 2, 9, 1, 7, 3, 3, 8, 1, 0, 4, 6], device=cuda)
    c1 = _cache(2, hkv, d, cuda)
    t1 = c1.new_sequence()
    full = model.forward(tokens, c1, t1)
    c2 = _cache(2, hkv, d, cuda)
    t2 = c2.new_sequence()
    for i in range(tokens.shape[0]):
        step = model.forward(tokens[i:i + 1], c2, t2)
    assert t1.length == t2.length == tokens.shape[0]
    torch.testing.assert_close(step[-1], full[-1], atol=3e-2, rtol=0)


def test_long_prefill_then_decode(cuda):
    """Prefill through the tcgen05 kernel (G*L > 64 rows), chunked prefill over a
    history (gather + prefill), then paged decode steps: each must agree with one
    full prefill of the same tokens."""
    import torch

    model = TinyDecoder(64, 64, 2, 8, 2, 64, 1024, cuda, seed=2)
    g = torch.Generator().manual_seed(5)
    tokens = torch.randint(0, 64, (300,), generator=g).to(cuda)
    c1 = _cache(2, 2, 64, cuda, blocks=128, bs=16)
    t1 = c1.new_sequence()
    full = model.forward(tokens, c1, t1)
    c2 = _cache(2, 2, 64, cuda, blocks=128, bs=16)
    t2 = c2.new_sequence()
    model.forward(tokens[:200], c2, t2)            # tcgen05 prefill
    model.forward(tokens[200:290], c2, t2)         # chunked prefill over a history
    for i in range(290, 300):                      # paged decode
        step = model.forward(tokens[i:i + 1], c2, t2)
    torch.testing.assert_close(step[-1], full[-1], atol=5e-2, rtol=0)


def _greedy(model, prompt, cache, n):
    import torch

    table = cache.new_sequence()
    logits = model.forward(torch.tensor(prompt, device=cache.device), cache, table)
    nxt = int(logits[-1].argmax())
    out = []
    for _ in range(n):
        out.append(nxt)
        logits = model.forward(torch.tensor([nxt], device=cache.device), cache, table)
        nxt = int(logits[-1].argmax())
    return out


def _speculative(target, draft, prompt, tcache, dcache, n, gamma):
    """Greedy speculative decoding (engine/decode/speculative.py:47-133 semantics)."""
    import torch

    dev = tcache.device
    tt, dt = tcache.new_sequence(), dcache.new_sequence()
    p = torch.tensor(prompt, device=dev)
    last = int(target.forward(p, tcache, tt)[-1].argmax())
    draft.forward(p, dcache, dt)
    out = [last]
    while len(out) < n:
        proposed, t = [], last
        for _ in range(gamma):
            t = int(draft.forward(torch.tensor([t], device=dev), dcache, dt)[-1].argmax())
            proposed.append(t)
        vl = target.forward(torch.tensor([last] + proposed, device=dev), tcache, tt)  # M = gamma+1
        accepted, fallback = 0, int(vl[0].argmax())
        for j in range(gamma):
            pred = int(vl[j].argmax())
            if pred == proposed[j]:
                accepted += 1
                fallback = int(vl[j + 1].argmax())
            else:
                fallback = pred
                break
        emitted = proposed[:accepted] + [fallback]
        keep = tt.length - (gamma - accepted)
        if keep < tt.length:
            tcache.rollback(tt, keep)
        keepd = dt.length - (gamma - accepted)
        if keepd < dt.length:
            dcache.rollback(dt, keepd)
        for tok in emitted:
            if len(out) >= n:
                break
            out.append(tok)
            last = tok
    return out


def test_speculative_matches_base_loop(cuda):
    target = TinyDecoder(32, 32, 2, 8, 2, 64, 256, cuda, seed=3)
    prompt = [1, 4, 2, 9, 11]
    base = _greedy(target, prompt, _cache(2, 2, 64, cuda), 12)
    spec = _speculative(target, target, prompt, _cache(2, 2, 64, cuda), _cache(2, 2, 64, cuda),
                        12, gamma=4)
    assert spec == base


@pytest.mark.parametrize("d", [64, 128])
def test_batched_step_matches_per_sequence(cuda, d):
    """begin_step + attention_forward_batch (one fused append and one attention
    launch for the whole batch, tables packed once per step) against
    attention_forward run sequence by sequence on a second cache: batched prefill
    of fresh prompts, then ragged histories through decode (L=1), speculative
    verify (L=5) and a chunked-prefill block (L=100)."""
    import torch

    from engine.attention import attention_forward, attention_forward_batch, begin_step
    from kernels import build_rope_cache

    hq, hkv = 8, 2
    rope = build_rope_cache(2048, d, theta=500000.0, device=cuda)
    g = torch.Generator().manual_seed(d)

    def rnd(*s):
        return torch.randn(*s, generator=g).to(cuda, torch.bfloat16)

    ca, cb = (_cache(1, hkv, d, cuda, blocks=160, bs=16) for _ in range(2))
    ta = [ca.new_sequence() for _ in range(3)]
    tb = [cb.new_sequence() for _ in range(3)]

    def run(L, what):
        q, k, v = rnd(3, hq, L, d), rnd(3, hkv, L, d), rnd(3, hkv, L, d)
        step = begin_step(ca, ta, L)
        out = attention_forward_batch(q, k, v, ca, 0, step, rope=rope)
        for b in range(3):
            ref = attention_forward(q[b:b + 1], k[b:b + 1], v[b:b + 1], cb, 0, tb[b], rope=rope)
            assert_close_attn(out[b:b + 1].float().cpu().numpy(), ref.float().cpu().numpy(),
                              what=f"{what} seq {b}")
        assert [t.length for t in ta] == [t.length for t in tb]

    run(96, "batched prefill")           # all histories empty: one tcgen05 launch
    for b, n in enumerate((0, 40, 171)):  # make the histories ragged
        if n:
            k, v = rnd(1, hkv, n, d), rnd(1, hkv, n, d)
            attention_forward(rnd(1, hq, n, d), k, v, ca, 0, ta[b], rope=rope)
            attention_forward(rnd(1, hq, n, d), k, v, cb, 0, tb[b], rope=rope)
    run(1, "decode")
    run(5, "verify")
    run(100, "chunked prefill")
    for b in range(3):
        ka, va = ca.gather(0, ta[b])
        kb, vb = cb.gather(0, tb[b])
        assert torch.equal(ka, kb) and torch.equal(va, vb)


@pytest.mark.parametrize("d", [64, 128])
def test_batched_step_vs_oracle(cuda, d):
    """The batched engine step against the oracle (not just against the CUDA
    per-sequence path): ragged histories (0, 40 and 171 tokens), then batch steps
    of decode (L=1), speculative verify (L=5), a chunked-prefill block (L=100,
    one tcgen05 launch reading the pools through the table) and decode again.
    The oracle keeps the raw K/V of every token, rotates K at its position (the
    cache stores rotated K, bf16-rounded, which the kernels reproduce bit for bit)
    and attends bottom-right causally with q rotated at its positions."""
    import torch

    import oracle
    from engine.attention import attention_forward, attention_forward_batch, begin_step
    from kernels import build_rope_cache
    from tests.golden.inputs import normal

    hq, hkv, B = 8, 2, 3
    c, s = oracle.build_rope_cache(2048, d, 500000.0)
    rope = build_rope_cache(2048, d, theta=500000.0, device=cuda)
    cache = _cache(1, hkv, d, cuda, blocks=160, bs=16)
    tables = [cache.new_sequence() for _ in range(B)]
    hist_k = [np.zeros((hkv, 0, d), np.float32) for _ in range(B)]
    hist_v = [np.zeros((hkv, 0, d), np.float32) for _ in range(B)]
    seed = [d * 100]

    def draw(shape):
        seed[0] += 1
        return normal(seed[0], shape)

    def remember(b, k, v, start):
        L = k.shape[1]
        krot = oracle.bf16_round(oracle.apply_rotary(k[None], c, s, np.arange(start, start + L))[0])
        hist_k[b] = np.concatenate([hist_k[b], krot], axis=1)
        hist_v[b] = np.concatenate([hist_v[b], v], axis=1)

    for b, n in enumerate((0, 40, 171)):
        if n:
            q, k, v = draw((1, hq, n, d)), draw((1, hkv, n, d)), draw((1, hkv, n, d))
            attention_forward(*(to_t(x, cuda) for x in (q, k, v)), cache, 0, tables[b], rope=rope)
            remember(b, k[0], v[0], 0)
    for L in (1, 5, 100, 1):
        q, k, v = draw((B, hq, L, d)), draw((B, hkv, L, d)), draw((B, hkv, L, d))
        step = begin_step(cache, tables, L)
        out = attention_forward_batch(*(to_t(x, cuda) for x in (q, k, v)), cache, 0, step,
                                      rope=rope).float().cpu().numpy()
        for b in range(B):
            start = step.starts[b]
            remember(b, k[b], v[b], start)
            qr = oracle.apply_rotary(q[b:b + 1], c, s, np.arange(start, start + L))
            ref = oracle.attention(qr, hist_k[b][None], hist_v[b][None], causal=True)
            assert_close_attn(out[b:b + 1], ref, what=f"L={L} seq {b} (history {start})")


def to_t(x, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(x)).to(device=device, dtype=torch.bfloat16)


def test_verify_loop_has_no_host_sync(cuda):
    """A speculative decoding round on the batched path — reserve and pack the
    tables for a verify block (begin_step), fused append + paged attention for every
    layer, roll the rejected drafts back, fork a sequence, then a decode step —
    runs with torch's sync debug mode set to raise on any host synchronisation:
    block tables reach the device through pinned non-blocking copies, the kernels
    are asynchronous, and rollback is host bookkeeping. The same device work of a
    step is then captured in a CUDA graph and replayed with the same result."""
    import torch

    from engine.attention import attention_forward_batch, begin_step
    from kernels import build_rope_cache

    hq, hkv, d, B, layers = 8, 2, 128, 3, 2
    rope = build_rope_cache(4096, d, theta=500000.0, device=cuda)
    cache = _cache(layers, hkv, d, cuda, blocks=256, bs=16)
    tables = [cache.new_sequence() for _ in range(B)]
    g = torch.Generator().manual_seed(11)

    def rnd(*s):
        return torch.randn(*s, generator=g).to(cuda, torch.bfloat16)

    prompt = [rnd(B, h, 300, d) for h in (hq, hkv, hkv)]
    verify = [rnd(B, h, 5, d) for h in (hq, hkv, hkv)]
    dec = [rnd(B, h, 1, d) for h in (hq, hkv, hkv)]
    step = begin_step(cache, tables, 300)
    for layer in range(layers):
        attention_forward_batch(*prompt, cache, layer, step, rope=rope)
    torch.cuda.synchronize()

    torch.cuda.set_sync_debug_mode("error")
    try:
        step = begin_step(cache, tables, 5)                     # verify block, M = gamma + 1
        outs = [attention_forward_batch(*verify, cache, layer, step, rope=rope)
                for layer in range(layers)]
        for t, accepted in zip(tables, (0, 2, 4)):              # rejected drafts roll back
            cache.rollback(t, t.length - (4 - accepted))
        forked = cache.fork(tables[1])
        step = begin_step(cache, tables, 1)                     # next decode step
        for layer in range(layers):
            attention_forward_batch(*dec, cache, layer, step, rope=rope)
    finally:
        torch.cuda.set_sync_debug_mode(0)
    torch.cuda.synchronize()
    assert forked.length == tables[1].length - 1
    assert all(torch.isfinite(o.float()).all() for o in outs)

    # the device work of one decode step as a CUDA graph
    step = begin_step(cache, tables, 1)
    eager = [attention_forward_batch(*dec, cache, layer, step, rope=rope)
             for layer in range(layers)]
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = [attention_forward_batch(*dec, cache, layer, step, rope=rope)
                    for layer in range(layers)]
    graph.replay()
    torch.cuda.synchronize()
    for a, b in zip(eager, captured):
        assert torch.equal(a, b)
