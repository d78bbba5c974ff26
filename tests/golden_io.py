"""Reads the golden vectors of tests/golden/ (written by the reference's own code, see
tests/golden/make_golden.cpp) into numpy arrays, one dict per case."""
import gzip
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
_DT = {"f32": np.float32, "f16": np.float16, "i8": np.int8, "i32": np.int32}


def load_golden():
    with open(os.path.join(GOLDEN, "golden.json")) as f:
        index = json.load(f)
    with gzip.open(os.path.join(GOLDEN, "golden.bin.gz"), "rb") as f:
        blob = f.read()
    cases = []
    for c in index["cases"]:
        case = {}
        for key, val in c.items():
            if isinstance(val, dict):
                dt = np.dtype(_DT[val["dtype"]])
                case[key] = np.frombuffer(blob, dtype=dt, count=val["bytes"] // dt.itemsize, offset=val["offset"]).copy()
            else:
                case[key] = val
        B, H, D = case["batch"], case["num_heads"], case["head_dim"]
        case["q"] = case["q"].reshape(B, H, D)
        case["ref"] = case["ref"].reshape(B, H, D)
        if "ref_fp32_data" in case:
            case["ref_fp32_data"] = case["ref_fp32_data"].reshape(B, H, D)
        Hkv = case["num_kv_heads"]
        if "page_size" in case:  # paged case: pools [num_blocks][Hkv][page][D]
            nb, P = case["num_blocks"], case["page_size"]
            case["k"] = case["k"][: nb * Hkv * P * D].reshape(nb, Hkv, P, D)
            case["v"] = case["v"][: nb * Hkv * P * D].reshape(nb, Hkv, P, D)
            case["block_table"] = case["block_table"].reshape(B, case["max_blocks"]) if B else case["block_table"]
            if "k_scale" in case:
                case["k_scale"] = case["k_scale"][: nb * Hkv].reshape(nb, Hkv)
                case["v_scale"] = case["v_scale"][: nb * Hkv].reshape(nb, Hkv)
        else:  # naive case: contiguous [B][Hkv][max_len][D]
            L = case["max_len"]
            case["k"] = case["k"].reshape(B, Hkv, L, D)
            case["v"] = case["v"].reshape(B, Hkv, L, D)
        for key in ("k32", "v32", "k_contig_f32", "v_contig_f32"):
            if key in case:
                case[key] = case[key].reshape(B, Hkv, case["max_len"], D)
        cases.append(case)
    return cases
