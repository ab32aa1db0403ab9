"""One quantized_matmul shape, timed with CUDA events (also the small case used for ncu
captures).  Usage:

    python bench_case.py M N K BITS [ACT|none] [REPS] [KERNEL] [LORA_RANK]

ACT: none, gelu_tanh, gelu or swiglu (a second W of the same shape as the up projection).
KERNEL: auto, gemm, gemm2, gemv, gemv_tc, gemv_tma, gemv_regs or generic.
LORA_RANK: r > 0 adds a LoRA adapter (A [K, r], B [r, N] ~N(0, 0.02), scale 0.5), fused.

Prints time per call and TFLOP/s / GB/s.
Weights ~N(0, 0.02) bf16 quantized on the device (group 64), x ~N(0, 1), bias ~N(0, 0.02).
"""
import os
import sys

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "mlx-gen_b200"))

import torch  # noqa: E402

import qlinear  # noqa: E402


def main(argv):
    M, N, K, bits = (int(v) for v in argv[:4])
    act = argv[4] if len(argv) > 4 and argv[4] != "none" else None
    reps = int(argv[5]) if len(argv) > 5 else 20
    kernel = {"gemm": qlinear.KERNEL_GEMM, "gemm2": qlinear.KERNEL_GEMM_PAIR, "gemv": qlinear.KERNEL_GEMV,
              "gemv_tc": qlinear.KERNEL_GEMV_TC, "gemv_tma": qlinear.KERNEL_GEMV_TMA,
              "gemv_regs": qlinear.KERNEL_GEMV_REGS, "generic": qlinear.KERNEL_GENERIC,
              "auto": qlinear.KERNEL_AUTO}[argv[6] if len(argv) > 6 else "auto"]
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(0)
    w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    bias = (torch.randn(N, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    wq, s, b = qlinear.quantize(w, 64, bits)
    del w
    up = None
    if act == "swiglu":
        w3 = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        up = qlinear.quantize(w3, 64, bits)
        del w3
    y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    rank = int(argv[7]) if len(argv) > 7 else 0
    lora = None
    if rank > 0:
        la = (torch.randn(K, rank, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        lb = (torch.randn(rank, N, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        lora = (la, lb, 0.5)

    def f():
        qlinear.quantized_matmul(x, wq, s, b, True, 64, bits, bias=bias, act=act, up=up, kernel=kernel, out=y,
                                 lora=lora)

    for _ in range(3):
        f()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        f()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    npass = 2 if act == "swiglu" else 1
    nbytes = npass * (N * K * bits // 8 + N * (K // 64) * 4) + (M * K + M * N) * 2
    print(f"M={M} N={N} K={K} Q{bits} act={act}{f' lora={rank}' if rank else ''}: {ms * 1e3:.1f} us  {2 * npass * M * N * K / ms / 1e9:.1f} TFLOP/s  "
          f"{nbytes / ms / 1e6:.1f} GB/s")


if __name__ == "__main__":
    main(sys.argv[1:])
