"""Generate the golden vectors in tests/golden/reference_golden.npz.

Runs the REFERENCE's own Python functions (src/w4a16/kernels.py of
emirabayer/w4a16-gemv-optimization-ladder: quantize_int4_symmetric,
quantize_int4_group, pack_int4, pack_int4_interleaved, dequant_ref,
dequant_ref_group, and benchmarks/perplexity.py's per-row fake-quant formula) on CPU
over small seeded inputs and stores inputs and outputs.  Run it where a checkout of
the reference is available, naming that checkout; the tests only read the .npz.

    python tests/golden/make_golden.py /path/to/reference
    W4A16_REFERENCE=/path/to/reference python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np
import torch

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("W4A16_REFERENCE")
if not REF:
    sys.exit("usage: make_golden.py /path/to/reference  (or set W4A16_REFERENCE)")
sys.path.insert(0, os.path.join(REF, "src"))
import w4a16 as R  # noqa: E402  (the reference package)

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_golden.npz")

# (name, rows, cols, weight std, special)
ROW_CASES = [
    ("row_16x256", 16, 256, 0.02, None),
    ("row_33x512", 33, 512, 0.02, None),       # rows not a multiple of 16
    ("row_8x2048", 8, 2048, 0.02, None),
    ("row_5x8", 5, 8, 0.02, None),             # smallest legal width
    ("row_3x24", 3, 24, 0.02, None),           # width not a multiple of 32
    ("row_12x512_n01", 12, 512, 1.0, None),    # N(0,1): the reference tests' weights
    ("row_32x1024_outlier", 32, 1024, 0.02, "outlier"),
    ("row_4x256_zero", 4, 256, 0.02, "zero"),  # one all-zero row
]
GROUP_CASES = [
    ("g128_16x256", 16, 256, 0.02, None),
    ("g128_33x512", 33, 512, 0.02, None),
    ("g128_8x2048", 8, 2048, 0.02, None),
    ("g128_4x128", 4, 128, 0.02, None),        # single group
    ("g128_12x512_n01", 12, 512, 1.0, None),
    ("g128_32x1024_outlier", 32, 1024, 0.02, "outlier"),
    ("g128_4x256_zero", 4, 256, 0.02, "zero"),  # one all-zero group
]


def weights(seed, rows, cols, std, special):
    torch.manual_seed(seed)
    w = torch.randn(rows, cols) * std
    if special == "outlier":  # 0.1% of weights scaled x20 (seeded index set)
        n = max(1, rows * cols // 1000)
        idx = torch.randperm(rows * cols)[:n]
        w.view(-1)[idx] *= 20.0
    w = w.half().float()  # fp16 weights, as the reference's benchmarks and tests use
    if special == "zero":
        if rows > 1:
            w[1] = 0.0
        w[0, :128] = 0.0
    x = torch.randn(cols).half()
    return w, x


def main():
    out = {}
    seed = 0
    kq = torch.tensor([[-4, -3, -2, -1, 0, 1, 2, 3]], dtype=torch.int8)
    out["known_q"] = kq.numpy()
    out["known_inter"] = R.pack_int4_interleaved(kq).numpy()
    out["known_simple"] = R.pack_int4(kq).numpy()
    names = []
    for group, cases in ((0, ROW_CASES), (128, GROUP_CASES)):
        for name, rows, cols, std, special in cases:
            w, x = weights(seed, rows, cols, std, special)
            seed += 1
            if group:
                q, s = R.quantize_int4_group(w, group=group)
                y = R.dequant_ref_group(q, s, x, group=group)
                s_full = s.repeat_interleave(group, dim=1)
            else:
                q, s = R.quantize_int4_symmetric(w)
                y = R.dequant_ref(q, s, x)
                s_full = s.unsqueeze(1)
            deq16 = (q.float() * s_full).half()
            out[f"{name}.w"] = w.half().numpy()  # exact: w is fp16-valued
            out[f"{name}.x"] = x.numpy()
            out[f"{name}.q"] = q.numpy()
            out[f"{name}.s"] = s.numpy()
            out[f"{name}.y"] = y.numpy()
            out[f"{name}.deq16"] = deq16.numpy()
            if cols % 8 == 0:
                out[f"{name}.inter"] = R.pack_int4_interleaved(q).numpy()
            out[f"{name}.simple"] = R.pack_int4(q).numpy()
            out[f"{name}.group"] = np.array(group)
            names.append(name)
    # per-row fake quant of benchmarks/perplexity.py:22-25 (q*scale in fp32, then fp16)
    w, _ = weights(1000, 16, 256, 0.02, None)
    scale = w.abs().max(dim=1, keepdim=True).values / 7.0
    qf = torch.round(w / scale).clamp(-8, 7)
    out["fakequant.w"] = w.half().numpy()
    out["fakequant.deq16"] = (qf * scale).to(w.dtype).half().numpy()
    out["cases"] = np.array(names)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {len(names)} cases, {os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    main()
