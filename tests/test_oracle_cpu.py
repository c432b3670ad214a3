"""The fp32 oracle that every kernel test compares against, checked against torch's SDPA:
paged causal GQA attention over a permuted block table with chunked-prefill query offsets
(the role of the reference's python/lake/engine/tests/test_torch_attention_backend.py:28,
which checks SDPA against a manual causal GQA computation)."""
import math

import torch
import torch.nn.functional as F

from lake_b200.oracle import ops_ref as ref


def test_paged_oracle_matches_sdpa_with_gqa_and_prefix_offsets():
    g = torch.Generator().manual_seed(0)
    hq, hkv, d, page, layers, layer = 8, 2, ref.HEAD_DIM, 16, 2, 1
    # (cached prefix, new query rows) per sequence: a fresh prompt, a chunk after a prefix, one decode row
    seqs = [(0, 37), (48, 20), (90, 1)]
    nblocks = sum((p + n + page - 1) // page for p, n in seqs) + 4
    arena = torch.zeros(nblocks, layers, 2, hkv, page, d)
    perm = torch.randperm(nblocks, generator=g).tolist()
    maxb = max((p + n + page - 1) // page for p, n in seqs)
    tables = torch.full((len(seqs), maxb), -1, dtype=torch.int32)
    ks, vs, qrows, qstart, pos = [], [], [], [0], []
    for s, (p, n) in enumerate(seqs):
        length = p + n
        nb = (length + page - 1) // page
        tables[s, :nb] = torch.tensor([perm.pop() for _ in range(nb)], dtype=torch.int32)
        k = torch.randn(length, hkv, d, generator=g)
        v = torch.randn(length, hkv, d, generator=g)
        slots = torch.tensor([int(tables[s, t // page]) * page + t % page for t in range(length)])
        ref.write_kv(arena, layer, slots, k, v)
        ks.append(k)
        vs.append(v)
        qrows.append(torch.randn(n, hq * d, generator=g))
        qstart.append(qstart[-1] + n)
        pos += list(range(p, length))
    q = torch.cat(qrows)
    lens = torch.tensor([p + n for p, n in seqs], dtype=torch.int32)
    scale = 1 / math.sqrt(d)
    got = ref.paged_attention(q, arena, layer, tables, lens, torch.tensor(qstart, dtype=torch.int32),
                              torch.tensor(pos, dtype=torch.int32), hq, hkv, scale)
    for s, (p, n) in enumerate(seqs):
        kk, vv = ref.gather_kv(arena, layer, tables[s], p + n)
        assert torch.equal(kk, ks[s]) and torch.equal(vv, vs[s])  # write/gather round trip
        qq = qrows[s].view(n, hq, d).transpose(0, 1)  # [Hq, n, D]
        kr = ks[s].repeat_interleave(hq // hkv, dim=1).transpose(0, 1)
        vr = vs[s].repeat_interleave(hq // hkv, dim=1).transpose(0, 1)
        visible = torch.arange(p + n)[None, :] <= torch.arange(p, p + n)[:, None]  # key j visible iff j <= pos
        want = F.scaled_dot_product_attention(qq, kr, vr, attn_mask=visible, scale=scale)
        torch.testing.assert_close(got[qstart[s]:qstart[s + 1]], want.transpose(0, 1).reshape(n, -1),
                                   atol=1e-5, rtol=1e-5)
