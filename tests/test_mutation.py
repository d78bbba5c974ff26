"""Mutation harness: known bugs planted one at a time, each of which the golden-vector checks must
catch. The reference's harness (scripts/mutation.sh:29-59) plants them in its GPU kernel and
expects its GPU tests to fail. On a shared GPU no kernel is broken on purpose, so the bugs are
planted in the CPU oracle (oracle/kvb_oracle.c, compiled from a mutated copy) instead. The checks are
the ones the CUDA kernels are checked against: the reference's own outputs within the kernel tolerance
(2e-5 absolute, NaN only where the reference has NaN), and its int8 pools and scales exactly. A
mutant that slips through means those checks could not tell that bug from a correct kernel either."""
import os
import subprocess

import numpy as np
import pytest

import oracle

TOL = 2e-5
SRC = os.path.join(os.path.dirname(oracle.__file__), "kvb_oracle.c")

# (bug, text in kvb_oracle.c, replacement); the same bug classes as the reference's list
MUTATIONS = [
    ("off-by-one row inside a page", "(size_t)(t % j->page)) * (size_t)j->D;",
     "(size_t)((t + 1) % j->page)) * (size_t)j->D;"),
    ("block table ignored (logical = physical)", "(size_t)j->table[(size_t)b * j->max_blocks + t / j->page];",
     "(size_t)(t / j->page);"),
    ("GQA: query head h reads KV head h % Hkv", "kvh = h / G,", "kvh = h % j->Hkv,"),
    ("no 1/sqrt(D) softmax scale", "const float scale = 1.0f / sqrtf((float)D);", "const float scale = 1.0f;"),
    ("last token left out of the weighted sum",
     "for (int t = 0; t < len; ++t) {\n            size_t slot;\n            const size_t off = row_offset(j, b, kvh, t, &slot);\n            const float vs",
     "for (int t = 0; t < len - 1; ++t) {\n            size_t slot;\n            const size_t off = row_offset(j, b, kvh, t, &slot);\n            const float vs"),
    ("empty sequence not 0", "len ? (float)(acc[d] / sum) : 0.0f", "(float)(acc[d] / sum)"),
    ("accumulator rounded to fp16 each token",
     "acc[d] += p[t] * load_elem(j->type, j->v, off + (size_t)d, vs);",
     "acc[d] = (double)(kvb_half)(acc[d] + p[t] * load_elem(j->type, j->v, off + (size_t)d, vs));"),
    ("int8: K scale not applied", "const float ks = j->type == KVB_ORACLE_I8 ? j->k_scale[slot] : 1.0f;",
     "const float ks = 1.0f;"),
    ("int8: scale of KV head 0 for every head", "*scale_slot = blk * (size_t)j->Hkv + (size_t)kvh;",
     "*scale_slot = blk * (size_t)j->Hkv;"),
    ("int8: V dequantized with the K scale", "j->v_scale[slot]", "j->k_scale[slot]"),
    ("quantizer rounds toward zero", "nearbyintf(x / scale)", "truncf(x / scale)"),
    ("quantizer scale = amax / 128", "const float scale = amax / 127.0f;", "const float scale = amax / 128.0f;"),
    ("quantizer writes every head's scale to head 0",
     "scales[(size_t)table[(size_t)b * max_blocks + i] * Hkv + kvh] = scale;",
     "scales[(size_t)table[(size_t)b * max_blocks + i] * Hkv] = scale;"),
]


def _golden_checks_pass(golden) -> bool:
    """True when the current oracle build passes every golden check the CUDA kernels face."""
    for c in golden:
        if "page_size" in c:
            out = oracle.paged_attention(c["q"], c["k"], c["v"], c["block_table"], c["seq_lens"],
                                         num_kv_heads=c["num_kv_heads"], page=c["page_size"], kv_type=c["kv_type"],
                                         k_scale=c.get("k_scale"), v_scale=c.get("v_scale"), threads=4)
            ref = c["ref"]
            if not np.array_equal(np.isnan(out), np.isnan(ref)):
                return False
            ok = ~np.isnan(ref)
            if ok.any() and np.abs(out[ok].astype(np.float64) - ref[ok]).max() > TOL:
                return False
        if "k_contig_f32" in c:
            for src, pool_key, scale_key in (("k_contig_f32", "k", "k_scale"), ("v_contig_f32", "v", "v_scale")):
                pool, scales = oracle.quantize_i8(c[src], c["block_table"], c["seq_lens"], num_blocks=c["num_blocks"],
                                                  page=c["page_size"])
                live = {int(c["block_table"][b, t // c["page_size"]])
                        for b, L in enumerate(c["seq_lens"]) for t in range(L)}
                for blk in live:
                    if not np.array_equal(scales[blk], c[scale_key][blk]):
                        return False
                for b, L in enumerate(c["seq_lens"]):
                    for t in range(L):
                        blk, r = c["block_table"][b, t // c["page_size"]], t % c["page_size"]
                        if not np.array_equal(pool[blk, :, r], c[pool_key][blk, :, r]):
                            return False
    return True


def test_unmutated_oracle_passes_the_checks(golden):
    assert _golden_checks_pass(golden)


@pytest.mark.parametrize("bug,old,new", MUTATIONS, ids=[m[0] for m in MUTATIONS])
def test_every_planted_bug_is_caught(golden, tmp_path, bug, old, new):
    src = open(SRC).read()
    assert src.count(old) == 1, f"mutation does not apply: {bug}"
    mutated = tmp_path / "kvb_oracle.c"
    mutated.write_text(src.replace(old, new))
    so = tmp_path / "liboracle_mutant.so"
    subprocess.run(["gcc", "-O2", "-std=c11", "-shared", "-fPIC", "-pthread", "-o", str(so), str(mutated), "-lm"],
                   check=True, capture_output=True)
    with oracle.use_library(str(so)):
        assert not _golden_checks_pass(golden), f"NOT CAUGHT: {bug}"
