"""The mutation harness against the CUDA kernels' own outputs.

The reference plants its kernel bugs in the GPU kernel and expects its GPU tests to fail
(scripts/mutation.sh:50-59). No kernel is broken on purpose on a shared GPU, so each bug is planted in
the CPU oracle (tests/test_mutation.py's list, compiled from a mutated copy of oracle/kvb_oracle.c)
and compared with what the unmodified CUDA kernels compute on the inputs the GPU tests use: the
golden vectors and a config-3-shaped int8 step. A kernel with that bug would compute the mutant's
output; the GPU tests compare the kernel with the correct oracle within 2e-5, so each mutant must
lie outside that tolerance of the real kernel's output on some input, or the GPU tests could not tell
the bug from a correct kernel. The quantizer bugs are checked the same way against the device
quantizer's pools (exact match required)."""
import subprocess

import numpy as np
import pytest
import torch

import kv_cache_bench_b200 as kvb
import oracle
from tests.cuda_runner import run_case
from tests.test_mutation import MUTATIONS, SRC

pytestmark = pytest.mark.gpu
TOL = 2e-5
DECODE_BUGS = [m for m in MUTATIONS if not m[0].startswith("quantizer")]
QUANT_BUGS = [m for m in MUTATIONS if m[0].startswith("quantizer")]


def _mutant(tmp_path, old, new):
    src = open(SRC).read()
    assert src.count(old) == 1
    (tmp_path / "kvb_oracle.c").write_text(src.replace(old, new))
    so = tmp_path / "liboracle_mutant.so"
    subprocess.run(["gcc", "-O2", "-std=c11", "-shared", "-fPIC", "-pthread", "-o", str(so),
                    str(tmp_path / "kvb_oracle.c"), "-lm"], check=True, capture_output=True)
    return str(so)


@pytest.fixture(scope="module")
def decode_cases(golden):
    """(inputs, CUDA output) for every paged golden case, plus a config-3-shaped int8 step with a
    second, shorter sequence and per-block magnitudes."""
    cases = []
    for c in golden:
        if "page_size" not in c:
            continue
        args = dict(q=c["q"], k=c["k"], v=c["v"], table=c["block_table"], lens=c["seq_lens"],
                    num_kv_heads=c["num_kv_heads"], page=c["page_size"], kv_type=c["kv_type"],
                    k_scale=c.get("k_scale"), v_scale=c.get("v_scale"))
        cases.append((args, run_case(c, part=c["part_tokens"])))
    big = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=[32768, 1000], kv_type=oracle.I8,
                           page=128, seed=3, varied=True)
    args = dict(q=big.q, k=big.k, v=big.v, table=big.table, lens=big.lens, num_kv_heads=8, page=128,
                kv_type=oracle.I8, k_scale=big.k_scale, v_scale=big.v_scale)
    cases.append((args, run_case(big)))
    return cases


def _oracle_out(a):
    return oracle.paged_attention(a["q"], a["k"], a["v"], a["table"], a["lens"], num_kv_heads=a["num_kv_heads"],
                                  page=a["page"], kv_type=a["kv_type"], k_scale=a["k_scale"], v_scale=a["v_scale"])


def test_unmutated_oracle_agrees_with_the_kernels(decode_cases):
    for a, out in decode_cases:
        assert oracle.max_abs_diff(out, _oracle_out(a)) <= TOL


@pytest.mark.parametrize("bug,old,new", DECODE_BUGS, ids=[m[0] for m in DECODE_BUGS])
def test_each_decode_bug_is_outside_the_kernel_tolerance(decode_cases, tmp_path, bug, old, new):
    worst = 0.0
    with oracle.use_library(_mutant(tmp_path, old, new)):
        for a, out in decode_cases:
            worst = max(worst, oracle.max_abs_diff(out, _oracle_out(a)))
            if worst > TOL:
                break
    assert worst > TOL, f"the kernel's output cannot tell this bug apart: {bug} ({worst:.3g})"


@pytest.mark.parametrize("bug,old,new", QUANT_BUGS, ids=[m[0] for m in QUANT_BUGS])
def test_each_quantizer_bug_differs_from_the_device_quantizer(tmp_path, bug, old, new):
    rng = np.random.default_rng(17)
    B, Hkv, D, page, lens = 2, 4, 128, 16, np.asarray([100, 37], np.int32)
    nblk = (lens + page - 1) // page
    num_blocks = int(nblk.sum()) + 3
    table, _ = oracle.layout_from_perm(lens, page, rng.permutation(num_blocks).astype(np.int32))
    contig = (rng.uniform(-1, 1, (B, Hkv, int(lens.max()), D)) *
              np.exp2(-rng.integers(0, 4, (B, Hkv, 1, 1)))).astype(np.float32)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    pool = torch.zeros((num_blocks, Hkv, page, D), dtype=torch.int8, device="cuda")
    scales = torch.zeros((num_blocks, Hkv), device="cuda")
    c, tb, ln = t(contig), t(table), t(lens)
    kvb.quantize_paged_i8(kvb.page_write_args(B, Hkv, D, kvb.KvType.i8, page, table.shape[1], int(lens.max()),
                                              contig=c.data_ptr(), block_table=tb.data_ptr(), seq_lens=ln.data_ptr(),
                                              pool=pool.data_ptr(), num_blocks=num_blocks, scales=scales.data_ptr()))
    gpu_pool, gpu_scales = pool.cpu().numpy(), scales.cpu().numpy()
    live = sorted({int(table[b, i]) for b in range(B) for i in range(int(nblk[b]))})
    ok_pool, ok_scales = oracle.quantize_i8(contig, table, lens, num_blocks=num_blocks, page=page)
    assert np.array_equal(ok_scales[live], gpu_scales[live])
    with oracle.use_library(_mutant(tmp_path, old, new)):
        m_pool, m_scales = oracle.quantize_i8(contig, table, lens, num_blocks=num_blocks, page=page)
    same = np.array_equal(m_scales[live], gpu_scales[live])
    for b in range(B):
        for tkn in range(int(lens[b])):
            blk, r = table[b, tkn // page], tkn % page
            same = same and np.array_equal(m_pool[blk, :, r], gpu_pool[blk, :, r])
    assert not same, f"the device quantizer's pool cannot tell this bug apart: {bug}"
