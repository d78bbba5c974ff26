"""The page write path on the GPU (kvb_quantize_paged_i8, kvb_scatter_paged) against the reference's
quantizer and scatter (src/reference.cpp:32-51, src/reference.hpp:60-68): the golden vectors the
reference's own code wrote, the pinned oracle on seeded inputs, exact round-half-to-even ties, zero
pages, slots that must stay untouched, bad lengths and block ids, a round trip through the decode
kernels, and size-independent properties at the int8 config's full size."""
import numpy as np
import pytest
import torch

import kv_cache_bench_b200 as kvb
import oracle

pytestmark = pytest.mark.gpu
SENTINEL = 0x55


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _gpu_write(contig, table, lens, *, num_blocks, page, kv_type, pool_fill=SENTINEL, error_word=None):
    contig = np.ascontiguousarray(contig)
    B, Hkv, max_len, D = contig.shape
    table = np.ascontiguousarray(table, np.int32).reshape(B, -1)
    dt = {oracle.F32: torch.float32, oracle.F16: torch.float16, oracle.I8: torch.int8}[kv_type]
    pool = torch.empty((num_blocks, Hkv, page, D), dtype=dt, device="cuda")
    pool.view(torch.uint8).fill_(pool_fill)
    scales = torch.full((num_blocks, Hkv), -1.0, device="cuda")
    c, tb, ln = _t(contig), _t(table), _t(np.asarray(lens, np.int32))
    a = kvb.page_write_args(B, Hkv, D, kvb.KvType(kv_type), page, table.shape[1], max_len, contig=c.data_ptr(),
                            block_table=tb.data_ptr(), seq_lens=ln.data_ptr(), pool=pool.data_ptr(),
                            num_blocks=num_blocks, scales=scales.data_ptr(),
                            error_word=error_word.data_ptr() if error_word is not None else 0)
    if kv_type == oracle.I8:
        kvb.quantize_paged_i8(a)
    else:
        kvb.scatter_paged(a)
    torch.cuda.synchronize()
    return pool.cpu().numpy(), scales.cpu().numpy()


def _live_slots(table, lens, page):
    for b, L in enumerate(lens):
        for t in range(int(L)):
            yield table[b, t // page], t % page


def _case(B_lens, Hkv, D, page, seed, slack=1.3):
    rng = np.random.default_rng(seed)
    lens = np.asarray(B_lens, np.int32)
    nblk = (lens + page - 1) // page
    num_blocks = max(1, int(np.ceil(nblk.sum() * slack)))
    table, _ = oracle.layout_from_perm(lens, page, rng.permutation(num_blocks).astype(np.int32))
    max_len = int(max(1, lens.max()))
    contig = rng.uniform(-1, 1, (len(lens), Hkv, max_len, D)).astype(np.float32)
    # magnitudes vary per 8-token run, so pages get different scales
    contig *= np.exp2(-rng.integers(0, 6, (len(lens), Hkv, (max_len + 7) // 8, 1)).repeat(8, 2)[:, :, :max_len])
    return contig, table, lens, num_blocks


def test_quantizer_reproduces_the_reference_golden_vectors(golden):
    n = 0
    for c in golden:
        if "k_contig_f32" not in c:
            continue
        for src, pool_key, scale_key in (("k_contig_f32", "k", "k_scale"), ("v_contig_f32", "v", "v_scale")):
            pool, scales = _gpu_write(c[src], c["block_table"], c["seq_lens"], num_blocks=c["num_blocks"],
                                      page=c["page_size"], kv_type=oracle.I8)
            live_blocks = {int(blk) for blk, _ in _live_slots(c["block_table"], c["seq_lens"], c["page_size"])}
            for blk in live_blocks:
                assert np.array_equal(scales[blk].view(np.uint32), c[scale_key][blk].view(np.uint32)), c["name"]
            for blk, r in _live_slots(c["block_table"], c["seq_lens"], c["page_size"]):
                assert np.array_equal(pool[blk, :, r], c[pool_key][blk, :, r]), c["name"]
            n += 1
    assert n >= 8


@pytest.mark.parametrize("page,D", [(16, 128), (64, 128), (128, 128), (256, 128), (8, 64), (32, 64)])
def test_quantizer_matches_oracle_bit_for_bit(page, D):
    contig, table, lens, num_blocks = _case([700, 0, 1, page, page + 1, 3 * page - 1], 4, D, page, seed=page + D)
    pool, scales = _gpu_write(contig, table, lens, num_blocks=num_blocks, page=page, kv_type=oracle.I8)
    ref_pool, ref_scales = oracle.quantize_i8(contig, table, lens, num_blocks=num_blocks, page=page)
    live = np.zeros(pool.shape[:3], bool)
    for blk, r in _live_slots(table, lens, page):
        live[blk, :, r] = True
    live_blocks = live.any(axis=(1, 2))
    assert np.array_equal(pool[live], ref_pool[live])
    assert np.array_equal(scales[live_blocks].view(np.uint32), ref_scales[live_blocks].view(np.uint32))
    # slots and blocks without a live token are not written
    assert (pool[~live].view(np.uint8) == SENTINEL).all()
    assert (scales[~live_blocks] == -1.0).all()


def test_quantizer_ties_round_half_to_even_and_zero_pages():
    page, D, Hkv = 16, 64, 2
    lens = [3 * page]
    table = np.arange(3, dtype=np.int32).reshape(1, 3)
    contig = np.zeros((1, Hkv, 3 * page, D), np.float32)
    # page 0: amax 127, so scale = 1 and x / scale hits every .5 tie
    ties = (np.arange(page * D, dtype=np.float32) % 254 - 127) + 0.5
    contig[0, :, :page] = np.clip(ties, -126.5, 126.5).reshape(page, D)
    contig[0, :, 0, 0] = 127.0
    # page 1: all zeros (scale 0, values 0); page 2: one tiny value
    contig[0, :, 2 * page + 3, 5] = 1e-30
    pool, scales = _gpu_write(contig, table, lens, num_blocks=3, page=page, kv_type=oracle.I8)
    ref_pool, ref_scales = oracle.quantize_i8(contig, table, lens, num_blocks=3, page=page)
    assert np.array_equal(pool, ref_pool) and np.array_equal(scales.view(np.uint32), ref_scales.view(np.uint32))
    assert scales[0, 0] == 1.0 and scales[1, 0] == 0.0
    x = contig[0, 0, 1, :8]
    assert np.array_equal(pool[0, 0, 1, :8], np.rint(x).astype(np.int8))  # 2.5 -> 2, 3.5 -> 4
    assert (pool[1] == 0).all()


@pytest.mark.parametrize("kv_type,page,D", [(oracle.F32, 16, 128), (oracle.F16, 64, 128), (oracle.F16, 8, 64),
                                            (oracle.F32, 256, 64)])
def test_scatter_matches_oracle(kv_type, page, D):
    contig, table, lens, num_blocks = _case([513, 0, 1, page, page + 1], 8, D, page, seed=7 * page + D)
    contig = contig.astype(oracle.NP_DTYPE[kv_type])
    pool, _ = _gpu_write(contig, table, lens, num_blocks=num_blocks, page=page, kv_type=kv_type)
    ref = oracle.scatter_paged(contig, table, lens, num_blocks=num_blocks, page=page)
    live = np.zeros(pool.shape[:3], bool)
    for blk, r in _live_slots(table, lens, page):
        live[blk, :, r] = True
    assert np.array_equal(pool[live].view(np.uint8), ref[live].view(np.uint8))
    assert (pool[~live].view(np.uint8) == SENTINEL).all()


def test_bad_lengths_and_block_ids_skip_the_page_and_flag():
    page, D = 16, 64
    contig, table, lens, num_blocks = _case([40, 40, 40], 2, D, page, seed=3)
    bad_lens = lens.copy()
    bad_lens[1] = 10_000  # more than max_len
    bad_table = table.copy()
    bad_table[2, 1] = num_blocks + 5  # refused block id
    word = torch.zeros(1, dtype=torch.int32, device="cuda")
    pool, _ = _gpu_write(contig, bad_table, bad_lens, num_blocks=num_blocks, page=page, kv_type=oracle.I8,
                         error_word=word)
    flag = int(word.item())
    assert flag & 1 and flag & 2
    ref_pool, _ = oracle.quantize_i8(contig, table, np.array([40, 0, 40], np.int32), num_blocks=num_blocks, page=page)
    for blk, r in _live_slots(table, [40, 0, 0], page):  # sequence 0 untouched by the errors
        assert np.array_equal(pool[blk, :, r], ref_pool[blk, :, r])
    for i in (0, 2):  # sequence 2: its good pages are written, the refused one is skipped
        blk = table[2, i]
        assert np.array_equal(pool[blk, :, : min(page, 40 - i * page)], ref_pool[blk, :, : min(page, 40 - i * page)])
    assert (pool[table[2, 1]].view(np.uint8) == SENTINEL).all()
    assert (pool[table[1, 0]].view(np.uint8) == SENTINEL).all()


def test_quantize_then_decode_equals_oracle_decode():
    """GPU-quantized pool -> GPU decode equals the fp64 oracle on the oracle-quantized pool."""
    page, D, Hkv, H = 64, 128, 8, 32
    kcon, table, lens, num_blocks = _case([3000, 77, 0, 1025], Hkv, D, page, seed=11)
    vcon = np.random.default_rng(12).uniform(-1, 1, kcon.shape).astype(np.float32)
    q = np.random.default_rng(13).uniform(-1, 1, (len(lens), H, D)).astype(np.float32)
    kp, ks = _gpu_write(kcon, table, lens, num_blocks=num_blocks, page=page, kv_type=oracle.I8, pool_fill=0)
    vp, vs = _gpu_write(vcon, table, lens, num_blocks=num_blocks, page=page, kv_type=oracle.I8, pool_fill=0)
    rk, rks = oracle.quantize_i8(kcon, table, lens, num_blocks=num_blocks, page=page)
    rv, rvs = oracle.quantize_i8(vcon, table, lens, num_blocks=num_blocks, page=page)
    ks[ks < 0] = 0
    vs[vs < 0] = 0
    ref = oracle.paged_attention(q, rk, rv, table, lens, num_kv_heads=Hkv, page=page, kv_type=oracle.I8,
                                 k_scale=rks, v_scale=rvs)
    from tests.cuda_runner import run_paged
    out = run_paged(q, kp, vp, table, lens, num_kv_heads=Hkv, page=page, kv_type=oracle.I8, k_scale=ks, v_scale=vs)
    assert oracle.max_abs_diff(out, ref) <= 2e-5


def test_full_size_quantization_properties():
    """Config 3's int8 cache (32768 tokens, 8 KV heads, page 128) quantized on the GPU: every page's
    scale is its max |x| / 127 and every live value is within half a scale step of its input."""
    B, Hkv, L, D, page = 1, 8, 32768, 128, 128
    g = torch.Generator(device="cuda").manual_seed(5)
    contig = torch.rand((B, Hkv, L, D), device="cuda", generator=g) * 2 - 1
    nb = L // page
    perm = torch.randperm(2 * nb, device="cuda", generator=g)[:nb].to(torch.int32).view(1, nb)
    lens = torch.tensor([L], dtype=torch.int32, device="cuda")
    pool = torch.zeros((2 * nb, Hkv, page, D), dtype=torch.int8, device="cuda")
    scales = torch.zeros((2 * nb, Hkv), device="cuda")
    a = kvb.page_write_args(B, Hkv, D, kvb.KvType.i8, page, nb, L, contig=contig.data_ptr(),
                            block_table=perm.data_ptr(), seq_lens=lens.data_ptr(), pool=pool.data_ptr(),
                            num_blocks=2 * nb, scales=scales.data_ptr())
    kvb.quantize_paged_i8(a)
    torch.cuda.synchronize()
    pages = contig.view(Hkv, nb, page, D).permute(1, 0, 2, 3)           # [nb][Hkv][page][D]
    blk = perm.view(-1).long()
    amax = pages.abs().amax(dim=(2, 3))
    # an IEEE fp32 division as in the reference (torch would multiply by a rounded 1/127)
    want = (amax.cpu().numpy() / np.float32(127.0)).astype(np.float32)
    assert np.array_equal(scales[blk].cpu().numpy().view(np.uint32), want.view(np.uint32))
    deq = pool[blk].float() * scales[blk][:, :, None, None]
    err = (deq - pages).abs() / scales[blk][:, :, None, None]
    assert float(err.max()) <= 0.5 + 1e-5
