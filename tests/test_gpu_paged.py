"""Paged KV caches (zllm_qkv_append_paged, zllm_attn_decode_paged): K and V pools of fixed-size pages
and a block table per sequence instead of one contiguous run per sequence.

* attention over pages scattered in random order (page sizes 16, 64 and 256, ragged lengths, f16 and
  f32, sequences sharing their prefix pages) gives the same bits as over a contiguous cache holding
  the same rows -- the split and the arithmetic are the contiguous kernel's;
* the paged append writes the same bits as the contiguous append, at the table's pages;
* a long context (32768 positions in 256-position pages) against the oracle within the f16-KV
  contract;
* a table entry out of range is reported (ZLLM_E_ARG at the next synchronization) instead of read.
"""
import numpy as np
import pytest

import oracle as O
from zerollm_b200.attention import (KVCache, PagedKV, attn_decode, attn_decode_paged, qkv_append, qkv_append_paged,
                                    rope_tables)
from zerollm_b200.kernels import Context
from zerollm_b200.lib import E_ARG, ZllmError

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
EPS = float(np.float32(1e-6))


@pytest.fixture(scope="module")
def ctx():
    c = Context(0)
    yield c
    c.close()


def _scatter(cache, layer, lens, page, rng, share_prefix=0):
    """A PagedKV holding the rows of `cache` (contiguous, layer `layer`) for sequences of `lens`, with
    pages in random pool order; with share_prefix > 0, sequence 1 points at sequence 0's first
    share_prefix pages (the caller makes those rows equal)."""
    nseq = len(lens)
    max_pages = (cache.max_ctx + page - 1) // page
    need = [(n + page - 1) // page for n in lens]
    total = sum(need) + 3                                   # a few unused pages in the pool
    order = rng.permutation(total)
    table = np.full((nseq, max_pages), -1, np.int32)
    it = iter(order)
    for s in range(nseq):
        for j in range(need[s]):
            table[s, j] = table[0, j] if (s == 1 and j < share_prefix) else next(it)
    table[table < 0] = 0                                    # entries past a sequence's length are never read
    kv = PagedKV(cache.ctx, cache.n_kv, cache.head_dim, total, page, cache.kv_f16, table)
    for s in range(nseq):
        for j in range(need[s]):
            p0, p1 = j * page, min(lens[s], (j + 1) * page)
            pg = int(table[s, j])
            kv.k[pg, :, :p1 - p0] = cache.t[s, layer, 0, :, p0:p1]
            kv.v[pg, :, :p1 - p0] = cache.t[s, layer, 1, :, p0:p1]
    return kv


CASES = [(16, True, (1, 17, 300)), (64, True, (2049, 64, 1000)), (256, False, (700, 1, 513)), (256, True, (5000, 4097))]


@pytest.mark.parametrize("page,kv_f16,lens", CASES)
def test_paged_attention_equals_contiguous(ctx, page, kv_f16, lens):
    rng = np.random.default_rng(page + len(lens) + kv_f16)
    nh, nkv, hd = 32, 8, 128
    L = max(lens) + 7
    cache = KVCache(ctx, 2, nkv, hd, L, kv_f16, len(lens))
    g = torch.Generator(device="cuda").manual_seed(page)
    vals = torch.randn(cache.t.shape, device="cuda", generator=g)
    cache.t.copy_(vals.half().view(torch.int16) if kv_f16 else vals)
    share = 2 if len(lens) > 1 and min(lens[0], lens[1]) >= 2 * page else 0
    if share:                                              # sequence 1 shares sequence 0's first pages
        cache.t[1, 1, :, :, :share * page] = cache.t[0, 1, :, :, :share * page]
    kv = _scatter(cache, 1, lens, page, rng, share_prefix=share)
    geo = cache.geom(nh, eps=EPS)
    q = torch.randn(len(lens), nh * hd, device="cuda", generator=g)
    npos = torch.as_tensor(np.array(lens, np.int32)).cuda()
    want = attn_decode(ctx, geo, cache, 1, q, npos, max(lens))
    got = attn_decode_paged(ctx, kv.geom(nh, eps=EPS), kv, q, npos, max(lens))
    ctx.sync()
    assert torch.equal(got, want)


@pytest.mark.parametrize("kv_f16", [True, False])
def test_paged_append_equals_contiguous(ctx, kv_f16):
    rng = np.random.default_rng(5 + kv_f16)
    nh, nkv, hd, page, L = 8, 2, 128, 16, 96
    cache = KVCache(ctx, 1, nkv, hd, L, kv_f16, 3)
    table = np.stack([rng.permutation(18)[:6] for _ in range(3)]).astype(np.int32)   # pages may repeat across rows:
    table[1] = np.arange(6, 12)                                                     # keep rows 0 / 2 disjoint from 1
    table[0] = np.arange(0, 6)
    table[2] = np.arange(12, 18)
    perm = rng.permutation(18)                                                      # then scatter the page ids
    table = perm[table].astype(np.int32)
    kv = PagedKV(ctx, nkv, hd, 18, page, kv_f16, table)
    ntok = 7
    q = torch.as_tensor((rng.standard_normal((ntok, nh * hd)) * 3).astype(np.float32)).cuda()
    k = torch.as_tensor((rng.standard_normal((ntok, nkv * hd)) * 3).astype(np.float32)).cuda()
    v = torch.as_tensor((rng.standard_normal((ntok, nkv * hd)) * 3).astype(np.float32)).cuda()
    qn = torch.as_tensor((1 + rng.standard_normal(hd) * 0.05).astype(np.float32)).cuda()
    kn = torch.as_tensor((1 + rng.standard_normal(hd) * 0.05).astype(np.float32)).cuda()
    pos_np = np.array([0, 15, 16, 33, 95, 47, 64], np.int32)
    seq_np = np.array([0, 1, 2, 0, 1, 2, 1], np.int32)
    pos, seq = torch.as_tensor(pos_np).cuda(), torch.as_tensor(seq_np).cuda()
    rope = rope_tables(ctx, hd, 1e6, L)
    geo = cache.geom(nh, eps=EPS)
    # the contiguous append writes every sequence's rows through cache.block(0, ...) + seq * seq_stride
    want_q = qkv_append(ctx, geo, cache, 0, q, k, v, pos, seq, rope, qn, kn)
    got_q = qkv_append_paged(ctx, kv.geom(nh, eps=EPS), kv, q, k, v, pos, seq, rope, qn, kn)
    ctx.sync()
    assert torch.equal(got_q, want_q)
    for t in range(ntok):
        s, p = int(seq_np[t]), int(pos_np[t])
        pg = int(table[s, p // page])
        assert torch.equal(kv.k[pg, :, p % page], cache.t[s, 0, 0, :, p])
        assert torch.equal(kv.v[pg, :, p % page], cache.t[s, 0, 1, :, p])


def test_paged_attention_long_context_matches_oracle(ctx):
    rng = np.random.default_rng(32768)
    nh, nkv, hd, page = 32, 8, 128, 256
    lens = (32768, 30001)
    cache = KVCache(ctx, 1, nkv, hd, max(lens), True, 2)
    g = torch.Generator(device="cuda").manual_seed(7)
    cache.t.copy_(torch.randn(cache.t.shape, device="cuda", generator=g).half().view(torch.int16))
    kv = _scatter(cache, 0, lens, page, rng)
    del cache
    q = torch.randn(2, nh * hd, device="cuda", generator=g)
    out = attn_decode_paged(ctx, kv.geom(nh, eps=EPS), kv, q, torch.as_tensor(np.array(lens, np.int32)).cuda(), max(lens))
    ctx.sync()
    out, qh, table = out.cpu().numpy(), q.cpu().numpy(), kv.table.cpu().numpy()
    for b, n in enumerate(lens):
        for h in (0, 21):
            kh = h // (nh // nkv)
            pages = table[b, :(n + page - 1) // page]
            K = torch.cat([kv.k[int(p), kh] for p in pages])[:n].cpu().numpy().view(np.uint16)
            V = torch.cat([kv.v[int(p), kh] for p in pages])[:n].cpu().numpy().view(np.uint16)
            want = O.attn_head(qh[b, h * hd:(h + 1) * hd], K, V, True)
            rel = float(np.abs(out[b, h * hd:(h + 1) * hd] - want).max() / np.abs(want).max())
            assert rel <= 2e-3, (b, h, rel)                 # the f16-KV contract
            assert rel <= 1e-5, (b, h, rel)


def test_paged_bad_table_entry_is_reported(ctx):
    nh, nkv, hd, page = 8, 2, 64, 16
    kv = PagedKV(ctx, nkv, hd, 4, page, True, np.array([[0, 1, 2, 7]], np.int32))   # page 7 of 4
    q = torch.randn(1, nh * hd, device="cuda")
    attn_decode_paged(ctx, kv.geom(nh), kv, q, torch.tensor([60], dtype=torch.int32, device="cuda"), 60)
    with pytest.raises(ZllmError, match="out of range") as e:
        ctx.sync()
    assert e.value.code == E_ARG
    ctx.sync()                                                # the context stays usable
    attn_decode_paged(ctx, kv.geom(nh), kv, q, torch.tensor([40], dtype=torch.int32, device="cuda"), 40)
    ctx.sync()
