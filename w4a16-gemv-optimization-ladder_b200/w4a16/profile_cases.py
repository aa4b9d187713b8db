"""Small, self-contained launches of single kernels, for profiler captures.

    python -m w4a16.profile_cases <case> [<case> ...]

Each case builds seeded random inputs (a few hundred MB on the device at most, always
larger than the 126 MB L2 so DRAM counters mean something), launches its kernel three
times and synchronises; the first launch is the warm-up, so a capture takes
`-k regex:<kernel> -s 1 -c 1`.  Cases:

    quantize_pack   fp16 65536 x 2048 -> simple packing, per-row scales  (k_quantize_pack)
    h2f32           lossy fp16-accumulate GEMV on 65536 x 2048            (k_h2f32)
    fp16_gemv       dense fp16 GEMV on 65536 x 2048                       (k_fp16_gemv)
    simple          per-row GEMV on the simple packing, 65536 x 2048      (k_gemv_tma, PACK 1)
    batch4          lm_head-sized 128256 x 2048 group-128, 4 vectors      (k_gemv_tma, NB 8)
    batch16         lm_head-sized 128256 x 2048 group-128, 16 vectors     (k_gemv_tma, NB 16, 6 warps)
    longk           down-projection-sized 8192 x 14336 group-128, 1 vector (k_gemv_tma, 9 warps)
    gemm            prefill: 2048 activation rows x 4096 x 4096, group-128 (k_gemm_tc)
    g128_f32        one vector, 65536 x 2048 group-128, fp32 scales    (k_gemv_tma)
    g128_f16        the same with fp16 scales                           (k_gemv_tma)
"""
import sys

import torch

from . import kernels as K

ROWS, COLS = 65536, 2048


def _weights(rows, cols, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(rows, cols, device="cuda", generator=g) * 0.02).half()
    x = torch.randn(cols, device="cuda", generator=g).half()
    return w, x


def _three(fn):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()


def case_quantize_pack():
    w, _ = _weights(ROWS, COLS, 0)
    _three(lambda: K.quantize_pack(w, group=0, packing="simple"))


def case_h2f32():
    w, x = _weights(ROWS, COLS, 1)
    p, s = K.quantize_pack(w, group=0, packing="simple")
    del w
    _three(lambda: K.matvec_h2f32(p, s, x))


def case_fp16_gemv():
    w, x = _weights(ROWS, COLS, 2)
    _three(lambda: K.matvec_fp16(w, x))


def case_simple():
    w, x = _weights(ROWS, COLS, 3)
    p, s = K.quantize_pack(w, group=0, packing="simple")
    del w
    _three(lambda: K.matvec_champ(p, s, x))


def _batched(rows, cols, batch, seed):
    w, _ = _weights(rows, cols, seed)
    p, s = K.quantize_pack(w, group=128)
    del w
    g = torch.Generator(device="cuda").manual_seed(seed + 100)
    x = torch.randn(batch, cols, device="cuda", generator=g).half() if batch > 1 else \
        torch.randn(cols, device="cuda", generator=g).half()
    _three(lambda: K.gemv(p, s, x, group=128))


def case_batch4():
    _batched(128256, 2048, 4, 4)


def case_batch16():
    _batched(128256, 2048, 16, 5)


def case_longk():
    _batched(8192, 14336, 1, 6)


def case_gemm():
    w, _ = _weights(4096, 4096, 7)
    p, s = K.quantize_pack(w, group=128)
    del w
    g = torch.Generator(device="cuda").manual_seed(107)
    x = torch.randn(2048, 4096, device="cuda", generator=g).half()
    _three(lambda: K.gemm(p, s, x, group=128))


def _g128(scale_dtype, seed):
    w, x = _weights(ROWS, COLS, seed)
    p, s = K.quantize_pack(w, group=128, scale_dtype=scale_dtype)
    del w
    _three(lambda: K.gemv(p, s, x, group=128))


def case_g128_f32():
    _g128(torch.float32, 8)


def case_g128_f16():
    _g128(torch.float16, 8)


CASES = {n[len("case_"):]: f for n, f in globals().items() if n.startswith("case_")}


def main(argv):
    if not argv or any(a not in CASES for a in argv):
        print(__doc__)
        return 2
    for a in argv:
        CASES[a]()
    print("ok")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
