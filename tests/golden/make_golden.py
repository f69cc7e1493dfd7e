"""Generate the golden vectors that pin the oracle to the reference implementation.

Run where the reference source is available (it is not on the GPU box):

    python tests/golden/make_golden.py --ref <reference checkout>/src

It imports the reference's own CPU path (``vllm_exact.kernels.digitize_torch`` / ``exact_linear_torch`` and
``vllm_exact.paged_attn.paged_decode_torch``), runs it on the seeded inputs of recipes.py, and writes:

* golden.json      sha256 of every output (and a few values for readability);
* attn_small.npz   the float32 attention outputs (compared with a tolerance, since float attention has no bit pin).
"""
import argparse
import importlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import recipes as R  # noqa: E402

ATTN_CASES = [  # (B, L, BS, H, KV, D, jitter): the reference test's first case and the BASELINE attention geometry
    (8, 300, 16, 16, 4, 256, False),
    (4, 200, 16, 32, 8, 128, True),
    (3, 1100, 528, 16, 4, 256, False),
]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference's src/ directory")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    K = importlib.import_module("vllm_exact.kernels")
    P = importlib.import_module("vllm_exact.paged_attn")
    torch.set_num_threads(8)
    gold = {"generator": "tests/golden/make_golden.py", "reference_functions": [
        "src/vllm_exact/kernels.py:22-39 digitize_torch", "src/vllm_exact/kernels.py:89-100 exact_linear_torch",
        "src/vllm_exact/paged_attn.py:117-132 paged_decode_torch"]}

    # configuration 1 (bf16 in, bf16 out)
    x, w = R.config1()
    xd, wd = K.digitize_torch(x.float(), 14), K.digitize_torch(w.float(), 14)
    y32 = K.exact_linear_torch(xd, wd, 14, True)
    y = y32.bfloat16()
    gold["config1"] = {"x_sha": R.sha(x), "w_sha": R.sha(w), "y_bf16_sha": R.sha(y), "y_f32_sha": R.sha(y32),
                       "y0_6": [float(v) for v in y[0, :6]], "sx": [int(v) for v in xd[3]],
                       "xd_sha": [R.sha(t) for t in xd], "wd_sha": [R.sha(t) for t in wd]}

    # the reference GPU test's shapes with extreme digits, both modes, fp32 and bf16 outputs
    cases = []
    for (M, N, Kd) in R.REF_GPU_SHAPES:
        x, w = R.extreme_digits(M, N, Kd)
        for F, tr in R.REF_GPU_MODES:
            xd, wd = K.digitize_torch(x, F), K.digitize_torch(w, F)
            ref = K.exact_linear_torch(xd, wd, F, tr)
            cases.append({"M": M, "N": N, "K": Kd, "F": F, "trunc": tr, "x_sha": R.sha(x), "w_sha": R.sha(w),
                          "xd_sha": [R.sha(t) for t in xd], "wd_sha": [R.sha(t) for t in wd],
                          "y_f32_sha": R.sha(ref), "y_bf16_sha": R.sha(ref.to(torch.bfloat16))})
    gold["extreme_digit_cases"] = cases

    # the reference CPU self-check fixture, all four (F, trunc) combinations
    x, w = R.ref_cpu_xw()
    gold["ref_cpu_xw"] = []
    for F in (14, 15):
        for tr in (False, True):
            y32 = K.exact_linear_torch(K.digitize_torch(x, F), K.digitize_torch(w, F), F, tr)
            gold["ref_cpu_xw"].append({"F": F, "trunc": tr, "y_f32_sha": R.sha(y32)})

    # digitizer: bf16 input of the reference GPU test, and the edge rows
    xb = R.digitize_bf16_input()
    gold["digitize_bf16"] = {"x_sha": R.sha(xb), "out": {str(F): [R.sha(t) for t in K.digitize_torch(xb.float(), F)]
                                                         for F in (14, 15)}}
    xe = R.digitize_edge_rows()
    gold["digitize_edge"] = {"x_sha": R.sha(xe), "out": {str(F): [R.sha(t) for t in K.digitize_torch(xe, F)]
                                                         for F in (14, 15)},
                             "sh": {str(F): [int(v) for v in K.digitize_torch(xe, F)[3]] for F in (14, 15)}}

    # attention: float outputs of the reference CPU oracle
    arrays = {}
    gold["attention"] = []
    for i, (B, L, BS, H, KV, D, jit) in enumerate(ATTN_CASES):
        q, kv, bt, sl = R.paged_case(B, L, BS, H, KV, D, ctx_jitter=jit)
        kc, vc = R.kv_views(kv, D)
        scale = 1.0 / D ** 0.5
        out = P.paged_decode_torch(q, kc, vc, bt, sl, scale, B)
        arrays[f"case{i}"] = out.numpy()
        gold["attention"].append({"B": B, "L": L, "BS": BS, "H": H, "KV": KV, "D": D, "jitter": jit, "scale": scale,
                                  "q_sha": R.sha(q), "kv_sha": R.sha(kv), "bt_sha": R.sha(bt), "sl_sha": R.sha(sl)})
    np.savez_compressed(HERE / "attn_small.npz", **arrays)
    (HERE / "golden.json").write_text(json.dumps(gold, indent=1) + "\n")
    print("wrote", HERE / "golden.json", HERE / "attn_small.npz")


if __name__ == "__main__":
    main()
