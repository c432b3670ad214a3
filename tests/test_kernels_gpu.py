"""Numerics of every sm_100a kernel against the fp32 PyTorch oracle (ops_ref)."""
import math

import pytest
import torch

from lake_b200 import ops
from lake_b200.oracle import ops_ref as ref
from lake_b200.ops.fp8 import quantize_blockwise, quantize_gate_up

pytestmark = pytest.mark.gpu

BF = torch.bfloat16


def _close(out, want, tol=2e-2):
    out = out.float()
    want = want.float()
    err = (out - want).abs().max().item()
    scale = want.abs().max().item() + 1e-6
    assert err <= tol * scale + 1e-3, f"max err {err} vs scale {scale}"


@pytest.mark.parametrize("m,n,k", [(1, 256, 64), (37, 512, 200), (128, 256, 4096), (300, 4096, 4096),
                                   (1024, 1024, 1024), (4096, 6144, 4096)])
def test_linear_bf16(cuda_dev, m, n, k):
    g = torch.Generator(device=cuda_dev).manual_seed(0)
    a = torch.randn(m, k, device=cuda_dev, generator=g).to(BF)
    w = (torch.randn(n, k, device=cuda_dev, generator=g) / math.sqrt(k)).to(BF)
    out = ops.linear(a, w)
    torch.cuda.synchronize()
    _close(out, ref.linear(a, w))
    ops.core.check_status()


def test_linear_f32_out(cuda_dev):
    a = torch.randn(200, 512, device=cuda_dev).to(BF)
    w = (torch.randn(768, 512, device=cuda_dev) / 20).to(BF)
    out = ops.linear(a, w, out_dtype=torch.float32)
    _close(out, ref.linear(a, w), 1e-2)


def test_linear_residual_inplace(cuda_dev):
    a = torch.randn(300, 1024, device=cuda_dev).to(BF)
    w = (torch.randn(512, 1024, device=cuda_dev) / 32).to(BF)
    h = torch.randn(300, 512, device=cuda_dev).to(BF)
    want = h.float() + ref.linear(a, w)
    ops.linear_residual(a, w, h, out=h)
    _close(h, want)


def test_linear_swiglu(cuda_dev):
    m, hdim, inter = 257, 512, 768
    a = torch.randn(m, hdim, device=cuda_dev).to(BF)
    gate = (torch.randn(inter, hdim, device=cuda_dev) / 20).to(BF)
    up = (torch.randn(inter, hdim, device=cuda_dev) / 20).to(BF)
    w = ref.interleave_gate_up(gate, up)
    out = ops.linear_swiglu(a, w)
    want = torch.nn.functional.silu(ref.linear(a, gate)) * ref.linear(a, up)
    _close(out, want)


def _arena(dev, blocks=64, layers=2, hkv=2):
    return torch.zeros(blocks, layers, 2, hkv, 16, 128, dtype=BF, device=dev)


@pytest.mark.parametrize("t", [70, 600])  # 600: two-SM kernel, two heads per 256-wide tile, ragged rows
def test_linear_qkv_rope_kv_write(cuda_dev, t):
    hid, hq, hkv = 512, 4, 2
    a = torch.randn(t, hid, device=cuda_dev).to(BF)
    w = (torch.randn((hq + 2 * hkv) * 128, hid, device=cuda_dev) / 20).to(BF)
    cs = ref.rope_cache(4096, 500000.0, device=cuda_dev)
    pos = torch.randint(0, 4000, (t,), device=cuda_dev, dtype=torch.int32)
    slots = torch.randperm(64 * 16, device=cuda_dev)[:t].to(torch.int64)
    slots[5] = -1
    arena = _arena(cuda_dev)
    arena_ref = arena.clone()
    q = torch.empty(t, hq * 128, dtype=BF, device=cuda_dev)
    ops.linear_qkv(a, w, q, cs, pos, slots, arena, 1, hq, hkv)
    # recompute the oracle on the GPU tensors for comparison
    acc = ref.linear(a, w)
    qq = ref.apply_rope(acc[:, : hq * 128].view(t, hq, 128), pos, cs).reshape(t, -1)
    kk = ref.apply_rope(acc[:, hq * 128:(hq + hkv) * 128].view(t, hkv, 128), pos, cs)
    vv = acc[:, (hq + hkv) * 128:].view(t, hkv, 128)
    ref.write_kv(arena_ref, 1, slots, kk, vv)
    torch.cuda.synchronize()
    _close(q, qq)
    _close(arena, arena_ref)


@pytest.mark.parametrize("m,vocab", [(3, 1024), (130, 128256)])
def test_linear_argmax(cuda_dev, m, vocab):
    a = torch.randn(m, 512, device=cuda_dev).to(BF)
    w = (torch.randn(vocab, 512, device=cuda_dev) / 20).to(BF)
    tok = ops.linear_argmax(a, w)
    logits = ops.linear(a, w, out_dtype=torch.float32)
    assert torch.equal(tok.cpu(), logits.argmax(-1).to(torch.int32).cpu())
    bm = torch.randint(-2**31, 2**31 - 1, (m, (vocab + 31) // 32), device=cuda_dev, dtype=torch.int32)
    tok2 = ops.linear_argmax(a, w, bitmask=bm)
    want = ref.greedy(logits, bm)
    assert torch.equal(tok2.cpu(), want.cpu())


def _fill_cache(dev, nseq, lens, hkv, layers=2, layer=1, blocks_per_seq=None):
    maxb = max((l + 15) // 16 for l in lens)
    bps = blocks_per_seq or maxb
    nblocks = nseq * bps + 3
    arena = (torch.randn(nblocks, layers, 2, hkv, 16, 128, device=dev) * 0.5).to(BF)
    perm = torch.randperm(nblocks, device=dev)[: nseq * bps].view(nseq, bps).to(torch.int32)
    return arena, perm


@pytest.mark.parametrize("nseq,hq,hkv,lens", [(3, 8, 2, [1, 17, 300]), (64, 32, 8, None), (2, 32, 8, [4096, 2000]),
                                             (5, 16, 8, [33, 64, 65, 128, 2])])
def test_paged_decode(cuda_dev, nseq, hq, hkv, lens):
    if lens is None:
        lens = torch.randint(1, 700, (nseq,)).tolist()
    arena, bt = _fill_cache(cuda_dev, nseq, lens, hkv)
    q = torch.randn(nseq, hq * 128, device=cuda_dev).to(BF)
    sl = torch.tensor(lens, dtype=torch.int32, device=cuda_dev)
    scale = 1 / math.sqrt(128)
    out = ops.paged_decode_attention(q, arena, 1, bt, sl, hq, hkv, scale)
    qs = torch.arange(nseq + 1, dtype=torch.int32, device=cuda_dev)
    want = ref.paged_attention(q, arena, 1, bt, sl, qs, sl - 1, hq, hkv, scale)
    torch.cuda.synchronize()
    _close(out, want)
    for splits in (1, 3):
        out2 = ops.paged_decode_attention(q, arena, 1, bt, sl, hq, hkv, scale, splits=splits)
        _close(out2, want)
    ops.core.check_status()


@pytest.mark.parametrize("hq,hkv,chunks", [(8, 2, [(0, 100)]), (32, 8, [(0, 2048)]),
                                           (16, 4, [(64, 37), (0, 1), (500, 200), (16, 64)]),
                                           (8, 8, [(0, 129), (130, 300), (1000, 5)])])
def test_paged_prefill(cuda_dev, hq, hkv, chunks):
    # chunks: (cached prefix length, new query tokens) per sequence
    lens = [p + n for p, n in chunks]
    arena, bt = _fill_cache(cuda_dev, len(chunks), lens, hkv)
    qstart = [0]
    pos0 = []
    positions = []
    for p, n in chunks:
        qstart.append(qstart[-1] + n)
        pos0.append(p)
        positions += list(range(p, p + n))
    t = qstart[-1]
    q = torch.randn(t, hq * 128, device=cuda_dev).to(BF)
    sl = torch.tensor(lens, dtype=torch.int32, device=cuda_dev)
    qs_t = torch.tensor(qstart, dtype=torch.int32, device=cuda_dev)
    pos_t = torch.tensor(positions, dtype=torch.int32, device=cuda_dev)
    scale = 1 / math.sqrt(128)
    want = ref.paged_attention(q, arena, 1, bt, sl, qs_t, pos_t, hq, hkv, scale)
    from lake_b200.ops._ext import native

    # tcgen05 with two heads per CTA (even GQA groups; default softmax and its variants 10-15),
    # tcgen05 with one head per CTA, warp MMA
    runs = [(True, 128, 1), (True, 128, 0), (False, 64, 1)] + [(True, 128, 10 + v) for v in range(6)]
    for tc, tile, kernel in runs:
        native().set_prefill_kernel(kernel)
        try:
            tiles = ops.build_prefill_tiles(qstart, pos0, tile=tile, device=cuda_dev)
            out = ops.paged_prefill_attention(q, arena, 1, bt, sl, tiles, qs_t, pos_t, hq, hkv, scale,
                                              tensor_core=tc)
            torch.cuda.synchronize()
        finally:
            native().set_prefill_kernel(1)
        _close(out, want)
    ops.core.check_status()


def test_paged_prefill_rescales_when_scores_grow(cuda_dev):
    """Keys whose scores jump by far more than 2^8 (log2 units) in later 128-key tiles force the
    two-head kernel's lazy O rescale; the result must still match the fp32 oracle."""
    hq, hkv, n = 8, 2, 700
    arena, bt = _fill_cache(cuda_dev, 1, [n], hkv)
    for page in range(arena.shape[0]):  # K grows with the page's position in the sequence
        pos = (bt[0] == page).nonzero()
        if pos.numel():
            arena[page, 1, 0] *= 1.0 + 1.5 * int(pos[0, 0]) / 8
    q = (torch.randn(n, hq * 128, device=cuda_dev) * 1.5).to(BF)
    sl = torch.tensor([n], dtype=torch.int32, device=cuda_dev)
    qs_t = torch.tensor([0, n], dtype=torch.int32, device=cuda_dev)
    pos_t = torch.arange(n, dtype=torch.int32, device=cuda_dev)
    scale = 1 / math.sqrt(128)
    want = ref.paged_attention(q, arena, 1, bt, sl, qs_t, pos_t, hq, hkv, scale)
    tiles = ops.build_prefill_tiles([0, n], [0], tile=128, device=cuda_dev)
    out = ops.paged_prefill_attention(q, arena, 1, bt, sl, tiles, qs_t, pos_t, hq, hkv, scale)
    torch.cuda.synchronize()
    _close(out, want)
    ops.core.check_status()


@pytest.mark.parametrize("rows,dim", [(1, 128), (300, 4096), (17, 8192), (64, 2048)])
def test_rmsnorm(cuda_dev, rows, dim):
    x = torch.randn(rows, dim, device=cuda_dev).to(BF)
    w = torch.rand(dim, device=cuda_dev).to(BF)
    _close(ops.rms_norm(x, w, 1e-5), ref.rms_norm(x, w, 1e-5))


def test_embedding(cuda_dev):
    table = torch.randn(1000, 512, device=cuda_dev).to(BF)
    ids = torch.randint(0, 1000, (77,), device=cuda_dev, dtype=torch.int32)
    assert torch.equal(ops.embedding(ids, table), table[ids.long()])


def test_greedy_bitmask_chain(cuda_dev):
    logits = torch.randn(9, 5000, device=cuda_dev)
    assert torch.equal(ops.greedy_sample(logits).cpu(), logits.argmax(-1).int().cpu())
    bm = torch.randint(-2**31, 2**31 - 1, (9, (5000 + 31) // 32), device=cuda_dev, dtype=torch.int32)
    assert torch.equal(ops.greedy_sample(logits, bm).cpu(), ref.greedy(logits, bm).cpu())
    l2 = logits.clone()
    ops.apply_token_bitmask(l2, bm)
    assert torch.equal(l2, ref.apply_bitmask(logits, bm))
    draft = torch.tensor([5, 6, 7, 1, 2], dtype=torch.int32, device=cuda_dev)
    doff = torch.tensor([0, 3, 5], dtype=torch.int32, device=cuda_dev)
    target = torch.tensor([5, 6, 9, 0, 1, 2, 8], dtype=torch.int32, device=cuda_dev)
    toff = torch.tensor([0, 4], dtype=torch.int32, device=cuda_dev)
    out, n = ops.chain_reject_sample(draft, doff, target, toff, 4)
    assert n.tolist() == [3, 3]
    assert out[0, :3].tolist() == [5, 6, 9] and out[1, :3].tolist() == [1, 2, 8]


def test_page_copy(cuda_dev):
    src = torch.randn(10, 4096, device=cuda_dev).to(BF)
    dst = torch.zeros(12, 4096, device=cuda_dev, dtype=BF)
    si = torch.tensor([3, 7, 1], device=cuda_dev)
    di = torch.tensor([0, 11, 5], device=cuda_dev)
    ops.page_copy(src, dst, si, di, 4096 * 2)
    assert torch.equal(dst[di], src[si])


@pytest.mark.parametrize("m,n,k", [(512, 4096, 4096), (777, 6144, 512), (1300, 2080, 1024), (4096, 28672, 4096)])
def test_gemm_pair_kernel_matches_fp32(cuda_dev, m, n, k):
    """Two-SM (cta_group::2) GEMM: plain store, residual, SwiGLU and fp32 epilogues vs fp32."""
    from lake_b200.ops._ext import native

    C = native()
    old = C.gemm_pair_mode()
    C.set_gemm_pair_mode(1)
    try:
        g = torch.Generator(device="cuda").manual_seed(m + n)
        a = (torch.randn(m, k, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
        w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).to(torch.bfloat16)
        want = a.float() @ w.float().t()
        out = ops.linear(a, w)
        assert (out.float() - want).abs().max().item() < 3e-2 * want.abs().max().item()
        out32 = ops.linear(a, w, out_dtype=torch.float32)
        assert (out32 - want).abs().max().item() < 1e-2 * want.abs().max().item()
        r = torch.randn(m, n, device="cuda", generator=g).to(torch.bfloat16)
        res = ops.linear_residual(a, w, r)
        assert (res.float() - (want + r.float())).abs().max().item() < 3e-2 * (want + r.float()).abs().max().item()
        if n % 256 == 0:
            act = ops.linear_swiglu(a, w)
            ref_act = ref.swiglu_from_interleaved(want)
            assert (act.float() - ref_act).abs().max().item() < 3e-2 * ref_act.abs().max().item() + 1e-3
        torch.cuda.synchronize()
        ops.core.check_status()
    finally:
        C.set_gemm_pair_mode(old)


@pytest.mark.parametrize("m,n,k", [(200, 4096, 14336), (64, 2048, 4096), (256, 4096, 4096)])
def test_gemm_split_k_small_m_matches_fp32(cuda_dev, m, n, k):
    """Small-M GEMMs split K across CTAs (fp32 workspace, last split applies the epilogue);
    repeated calls check the workspace is left zeroed."""
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n)
    a = (torch.randn(m, k, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).to(torch.bfloat16)
    r = torch.randn(m, n, device="cuda", generator=g).to(torch.bfloat16)
    want = a.float() @ w.float().t()
    for _ in range(3):
        out = ops.linear(a, w)
        assert (out.float() - want).abs().max().item() < 3e-2 * want.abs().max().item()
        res = ops.linear_residual(a, w, r)
        assert (res.float() - (want + r.float())).abs().max().item() < 3e-2 * (want + r.float()).abs().max().item()
        o32 = ops.linear(a, w, out_dtype=torch.float32)
        assert (o32 - want).abs().max().item() < 1e-2 * want.abs().max().item()
        if n % 256 == 0:
            act = ops.linear_swiglu(a, w)
            ref_act = ref.swiglu_from_interleaved(want)
            assert (act.float() - ref_act).abs().max().item() < 3e-2 * ref_act.abs().max().item() + 1e-3
    torch.cuda.synchronize()
    ops.core.check_status()


@pytest.mark.parametrize("m,n,k", [(300, 1024, 512), (64, 4096, 4096), (2048, 2304, 1024)])
def test_gemm_fp8_weights_match_dequantized(cuda_dev, m, n, k):
    """W8A16: block-scaled e4m3 weights dequantised in shared memory by converter warps (the W8A8
    path is switched off here; it has its own test)."""
    from lake_b200.ops._ext import native

    native().set_gemm_w8a8_min_m(0)
    try:
        _fp8_weights_case(m, n, k)
    finally:
        native().set_gemm_w8a8_min_m(256)


def _fp8_weights_case(m, n, k):

    g = torch.Generator(device="cuda").manual_seed(m + k)
    a = (torch.randn(m, k, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    w = torch.randn(n, k, device="cuda", generator=g) / k ** 0.5
    w[:128, :128] *= 40.0  # blocks with very different scales
    w8 = quantize_blockwise(w)
    wd = w8.dequant().to(torch.bfloat16).float()  # the kernel rounds value x scale to bf16
    want = a.float() @ wd.t()
    tol = 2e-2 * want.abs().max().item()
    out = ops.linear(a, w8)
    assert (out.float() - want).abs().max().item() < tol
    r = torch.randn(m, n, device="cuda", generator=g).to(torch.bfloat16)
    res = ops.linear_residual(a, w8, r)
    assert (res.float() - (want + r.float())).abs().max().item() < tol + 2e-2
    if n % 256 == 0:
        gu8 = quantize_gate_up(w)  # fp8 SwiGLU weights: gate/up interleaved per 128 rows
        gu_want = a.float() @ gu8.dequant().to(torch.bfloat16).float().t()
        act = ops.linear_swiglu(a, gu8)
        ref_act = ref.swiglu_from_interleaved(gu_want, 128)
        assert (act.float() - ref_act).abs().max().item() < 3e-2 * ref_act.abs().max().item() + 1e-3
    toks = ops.linear_argmax(a, w8)
    assert (toks.long().cpu() == want.argmax(-1).cpu()).float().mean().item() > 0.97
    torch.cuda.synchronize()
    ops.core.check_status()


@pytest.mark.parametrize("m,n,k", [(300, 1024, 512), (1000, 2304, 1024), (4096, 6144, 4096)])
def test_gemm_w8a8_matches_quantized_operands(cuda_dev, m, n, k):
    """W8A8: the activations quantised to e4m3 per row and 128-column block, kind::f8f6f4 MMAs per
    128-deep k-block, each k-block's product scaled by its two block scales in fp32. Equal to the
    fp32 product of the dequantised operands up to the bf16 output rounding; the kernel's
    quantisation equal to the PyTorch restatement of it."""
    from lake_b200.ops._ext import native
    from lake_b200.ops.fp8 import quantize_rows

    C = native()
    C.set_gemm_w8a8_min_m(1)
    try:
        assert C.gemm_w8a8_reserve(m, k)
        g = torch.Generator(device="cuda").manual_seed(m + n)
        a = (torch.randn(m, k, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
        a[:7, :128] *= 30.0  # activation blocks with very different scales
        w = torch.randn(n, k, device="cuda", generator=g) / k ** 0.5
        w[:128, :128] *= 40.0
        w8 = quantize_blockwise(w)
        aq, asc = quantize_rows(a)
        q = torch.empty(m, k, dtype=torch.uint8, device="cuda")
        s = torch.empty(m, k // 128, dtype=torch.float32, device="cuda")
        C.quantize_fp8_rows(a, q, s)
        assert torch.equal(s, asc)
        assert (q.view(torch.float8_e4m3fn).float() == aq).float().mean().item() > 0.9999
        ad = (aq.view(m, k // 128, 128) * asc[..., None]).view(m, k)
        want = ad @ w8.dequant().t()
        tol = 1e-2 * want.abs().max().item()
        assert (ops.linear(a, w8).float() - want).abs().max().item() < tol
        r = torch.randn(m, n, device="cuda", generator=g).to(torch.bfloat16)
        res = ops.linear_residual(a, w8, r)
        assert (res.float() - (want + r.float())).abs().max().item() < tol + 2e-2
        if n % 256 == 0:
            gu8 = quantize_gate_up(w)
            act = ops.linear_swiglu(a, gu8)
            ref_act = ref.swiglu_from_interleaved(ad @ gu8.dequant().t(), 128)
            assert (act.float() - ref_act).abs().max().item() < 2e-2 * ref_act.abs().max().item() + 1e-3
        toks = ops.linear_argmax(a, w8)
        assert (toks.long().cpu() == want.argmax(-1).cpu()).float().mean().item() > 0.97
        torch.cuda.synchronize()
        ops.core.check_status()
    finally:
        C.set_gemm_w8a8_min_m(256)


@pytest.mark.parametrize("m", [1024, 1000, 8192])
def test_qkv_peer_kv_stores_equal_local(cuda_dev, m):
    """Fused P->D: the QKV epilogue's K/V rows written into a second GPU's arena over NVLink
    (coalesced through shared memory in the two-SM kernel) are bit-identical to the local
    arena's, with slots that cross pages and a ragged last tile."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from lake_b200.ops._ext import native

    native().enable_peer_access(1)
    hq, hkv, hidden = 32, 8, 4096
    nb = (m + 15) // 16 + 8
    arena = torch.zeros(nb, 2, 2, hkv, 16, 128, device=cuda_dev, dtype=BF)
    peer = torch.zeros(nb, 2, 2, hkv, 16, 128, device="cuda:1", dtype=BF)
    x = torch.randn(m, hidden, device=cuda_dev).to(BF)
    w = (torch.randn((hq + 2 * hkv) * 128, hidden, device=cuda_dev) * 0.02).to(BF)
    q = torch.empty(m, hq * 128, device=cuda_dev, dtype=BF)
    cs = ref.rope_cache(8192, 5e5, 128, None, device=cuda_dev)
    pos = torch.arange(m, dtype=torch.int32, device=cuda_dev) + 7
    slots = torch.randperm(nb * 16, device=cuda_dev)[:m].to(torch.int64)  # scattered over pages
    pslots = (slots + 16 * 3) % (nb * 16)  # a different placement in the peer arena
    ops.linear_qkv(x, w, q, cs, pos, slots, arena, 1, hq, hkv, peer, pslots)
    torch.cuda.synchronize()
    ops.core.check_status()
    flat_l = arena[:, 1].permute(0, 3, 1, 2, 4).reshape(nb * 16, 2, hkv, 128)  # [slot, k/v, head, dim]
    flat_p = peer[:, 1].permute(0, 3, 1, 2, 4).reshape(nb * 16, 2, hkv, 128).to(cuda_dev)
    assert torch.equal(flat_l[slots], flat_p[pslots])
    assert flat_l[slots].abs().sum().item() > 0
