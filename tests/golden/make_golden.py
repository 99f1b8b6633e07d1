"""Generate the golden NF4-unpack vectors from the reference kernel itself.

Runs the reference's Triton kernel `_nf4_unpack` (solution/nf4.py:30-50, launched
by `dequantize_nf4`, nf4.py:73-92) under the Triton CPU interpreter
(TRITON_INTERPRET=1) on seeded inputs, and stores inputs + outputs (small cases)
or their SHA-256 digests (large cases) in nf4_golden.npz / nf4_golden.json.

bitsandbytes (the reference's source of the NF4 table, nf4.py:53-58) is absent
here, so the table is injected into the reference module's `_CODE` cache; the
inputs come from oracle.nf4_oracle.quantize_nf4 (seeded).  This pins the decode
arithmetic (scale, nibble order, rounding) to the reference kernel; the codebook
values are inputs of that arithmetic.

Run from the repo root, in an environment that has the reference checkout:
    python tests/golden/make_golden.py [path/to/reference]
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys
import time

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import nf4_oracle as O  # noqa: E402

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("STEW_REFERENCE")
if not REF:
    sys.exit("usage: make_golden.py <path to the reference checkout> (or set STEW_REFERENCE)")

# (name, shape, blocksize, nested, out dtype, store full arrays?, input kind)
CASES = [
    ("edge_100x64_bs64_nested", (100, 64), 64, True, "float16", True, "normal"),
    ("edge_100x64_bs64_plain", (100, 64), 64, False, "float16", True, "normal"),
    ("edge_100x64_bs128_nested", (100, 64), 128, True, "float16", True, "normal"),
    ("edge_100x64_bs128_plain", (100, 64), 128, False, "float16", True, "normal"),
    ("kv_256x1536_bs64_nested", (256, 1536), 64, True, "float16", False, "normal"),
    ("kv_256x1536_bs64_plain", (256, 1536), 64, False, "float16", False, "normal"),
    ("kv_256x1536_bs128_nested", (256, 1536), 128, True, "float16", False, "normal"),
    ("q_1536x1536_bs64_nested", (1536, 1536), 64, True, "float16", False, "normal"),
    ("q_1536x1536_bs64_plain", (1536, 1536), 64, False, "float16", False, "normal"),
    ("small_64x512_bs32_nested", (64, 512), 32, True, "float16", True, "normal"),
    ("small_64x512_bs256_nested", (64, 512), 256, True, "float16", True, "normal"),
    ("small_128x512_bs64_nested_f32", (128, 512), 64, True, "float32", True, "normal"),
    ("small_128x512_bs64_plain_f32", (128, 512), 64, False, "float32", True, "normal"),
    # every byte value, every 8-bit absmax code, wide second-level scales and a
    # large offset: overflow to inf and fp16 subnormals are both reached
    ("rand_bytes_256x512_bs64_nested", (256, 512), 64, True, "float16", True, "random"),
    ("rand_bytes_256x512_bs64_plain", (256, 512), 64, False, "float16", True, "random"),
]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def make_inputs(shape, bs, nested, dtype, kind, seed):
    return O.golden_inputs(shape, bs, nested, dtype, kind, seed)


class _S2:
    pass


class _St:
    pass


def to_ref_state(st: O.QState):
    """A duck-typed QuantState with the attributes nf4.py:61-91 reads, on CPU tensors."""
    r = _St()
    r.shape = torch.Size(st.shape)
    r.dtype = torch.float16 if st.dtype == "float16" else torch.float32
    r.blocksize = st.blocksize
    r.quant_type = "nf4"
    r.nested = st.nested
    r.absmax = torch.from_numpy(np.ascontiguousarray(st.absmax))
    if st.nested:
        r.offset = torch.tensor(st.offset, dtype=torch.float32)
        s2 = _S2()
        s2.code = torch.from_numpy(st.state2.code.copy())
        s2.absmax = torch.from_numpy(st.state2.absmax.copy())
        s2.blocksize = st.state2.blocksize
        r.state2 = s2
    return r


def main():
    spec = importlib.util.spec_from_file_location("ref_nf4", os.path.join(REF, "solution", "nf4.py"))
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    ref._CODE["cpu"] = torch.from_numpy(O.nf4_codebook())

    arrays, meta = {}, {"generator": "reference solution/nf4.py _nf4_unpack under TRITON_INTERPRET=1",
                        "codebook": "QLoRA paper Appendix E NF4 table (oracle.nf4_oracle.NF4_PUBLISHED)",
                        "code2": "oracle.nf4_oracle.dynamic_map_signed()",
                        "cases": []}
    for i, (name, shape, bs, nested, dtype, full, kind) in enumerate(CASES):
        seed = 1000 + i
        packed, st = make_inputs(shape, bs, nested, dtype, kind, seed)
        t0 = time.time()
        out = ref.dequantize_nf4(torch.from_numpy(packed), to_ref_state(st)).numpy()
        dt = time.time() - t0
        mine = O.dequant_nf4(packed, st)
        same = bool(np.array_equal(out.view(np.uint16 if dtype == "float16" else np.uint32),
                                   mine.view(np.uint16 if dtype == "float16" else np.uint32)))
        print(f"{name:36s} ref {dt:6.2f}s  oracle bit-identical: {same}")
        case = {"name": name, "shape": list(shape), "blocksize": bs, "nested": nested, "dtype": dtype,
                "kind": kind, "seed": seed, "full": full, "offset": float(st.offset),
                "sha_packed": sha(packed), "sha_absmax": sha(np.asarray(st.absmax)),
                "sha_out": sha(out), "oracle_matches_at_generation": same}
        if nested:
            case["sha_absmax2"] = sha(st.state2.absmax)
        meta["cases"].append(case)
        if full:
            arrays[f"{name}/packed"] = packed
            arrays[f"{name}/absmax"] = np.asarray(st.absmax)
            arrays[f"{name}/out"] = out
            if nested:
                arrays[f"{name}/absmax2"] = st.state2.absmax
    arrays["code"] = O.nf4_codebook()
    arrays["code2"] = O.dynamic_map_signed()
    np.savez_compressed(os.path.join(HERE, "nf4_golden.npz"), **arrays)
    with open(os.path.join(HERE, "nf4_golden.json"), "w") as f:
        json.dump(meta, f, indent=1)


if __name__ == "__main__":
    main()
