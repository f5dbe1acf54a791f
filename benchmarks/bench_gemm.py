"""Local GEMM benchmark: the tcgen05 kernels against cuBLAS (torch.matmul).

Layouts follow the einsum canonicaliser's naming: ``a_mn``/``b_mn`` say
whether A/B are MN-major in memory (A stored [K][M], B stored [K][N]).  The
TP-MLP config produces all four: forward NT (both K-major), backward dX NN
(B MN-major) and dW TN-style (both MN-major).

Two modes:
  burst      CUDA events per iteration (inputs larger than L2 at the default
             sizes, so no flush is needed)
Kernels: cublas, 1sm, 2sm, wide (one pair tile per cluster), widep (wide,
persistent clusters), streamk (wide, every tile split), auto (the heuristics:
stream-K tail for the partial last wave of long-K GEMMs).

  sustained  back-to-back launches for --seconds while nvidia-smi samples SM
             clock and power; reports TFLOP/s with the median clock/power, the
             regime in which a long training step runs under the 1 kW cap

    python benchmarks/bench_gemm.py --mode sustained --kernels cublas,1sm,2sm
"""

import statistics
import subprocess
import threading
import time

import torch

from common import Writer, benchmark, parser, peaks

SHAPES = {
    # name: (M, N, K, a_mn, b_mn)
    "tp_fwd_nt": (32768, 28672, 8192, 0, 0),
    "tp_dx_nn": (32768, 8192, 28672, 0, 1),
    "tp_dw_tt": (28672, 8192, 32768, 1, 1),
    "cube_nt": (8192, 8192, 8192, 0, 0),
    "cube_nn": (8192, 8192, 8192, 0, 1),
    "cube_tt": (8192, 8192, 8192, 1, 1),
    # transformer training config (65536 tokens per rank, d=2048, MLP 8192, vocab 32000):
    # forward x W^T, input gradient dY W, weight gradient dY^T x
    "tr_d_fwd": (65536, 2048, 2048, 0, 0),
    "tr_up_fwd": (65536, 8192, 2048, 0, 0),
    "tr_dn_fwd": (65536, 2048, 8192, 0, 0),
    "tr_d_dx": (65536, 2048, 2048, 0, 1),
    "tr_up_dx": (65536, 2048, 8192, 0, 1),
    "tr_dn_dx": (65536, 8192, 2048, 0, 1),
    "tr_d_dw": (2048, 2048, 65536, 1, 1),
    "tr_up_dw": (8192, 2048, 65536, 1, 1),
    "tr_dn_dw": (2048, 8192, 65536, 1, 1),
    "tr_head_fwd": (65536, 32000, 2048, 0, 0),
    "tr_head_dw": (32000, 2048, 65536, 1, 1),
    # TP-MLP at tp=8 (h/tp = 3584): weight gradient with 224 pair tiles
    "tp8_dw_tt": (3584, 8192, 32768, 1, 1),
}


def make_operands(m, n, k, a_mn, b_mn, device):
    g = torch.Generator(device=device).manual_seed(0)
    a = (torch.randn(k, m, device=device, dtype=torch.bfloat16, generator=g).t() if a_mn
         else torch.randn(m, k, device=device, dtype=torch.bfloat16, generator=g))
    b = (torch.randn(k, n, device=device, dtype=torch.bfloat16, generator=g) if b_mn
         else torch.randn(n, k, device=device, dtype=torch.bfloat16, generator=g).t())
    return a.unsqueeze(0), b.unsqueeze(0)


class Sampler:
    def __init__(self):
        self.samples, self._stop = [], threading.Event()

    def _run(self):
        while not self._stop.is_set():
            out = subprocess.run(["nvidia-smi", "-i", str(torch.cuda.current_device()),
                                  "--query-gpu=clocks.sm,power.draw", "--format=csv,noheader,nounits"],
                                 capture_output=True, text=True).stdout.strip()
            try:
                mhz, watts = (float(v) for v in out.split(","))
                self.samples.append((mhz, watts))
            except ValueError:
                pass
            time.sleep(0.1)

    def __enter__(self):
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self.thread.join()
        return False


def sustained(fn, seconds):
    fn()
    torch.cuda.synchronize()
    # queue a bounded number of launches per chunk so the host never runs far ahead
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    while time.time() - t0 < 0.5:
        fn()
        torch.cuda.synchronize()
    n = 0
    with Sampler() as s:
        start.record()
        t0 = time.time()
        while time.time() - t0 < seconds:
            for _ in range(4):
                fn()
            n += 4
            torch.cuda.synchronize()
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / n
    mhz = statistics.median(x[0] for x in s.samples) if s.samples else None
    watts = statistics.median(x[1] for x in s.samples) if s.samples else None
    return ms, mhz, watts


def main():
    p = parser(__doc__)
    p.add_argument("--mode", choices=("burst", "sustained"), default="burst")
    p.add_argument("--seconds", type=float, default=2.0)
    p.add_argument("--shapes", default="cube_nt,cube_nn,cube_tt")
    p.add_argument("--kernels", default="cublas,1sm,2sm")
    p.add_argument("--group-m", type=int, default=0)
    p.add_argument("--split", type=int, default=0, help="wide kernel: cluster split mode 0/1/2")
    p.add_argument("--sleep-ns", type=int, default=0, help="wide kernel: epilogue back-off between polls")
    p.add_argument("--l2-promotion", type=int, default=3, help="TMA L2 promotion 0 none .. 3 256B")
    p.add_argument("--persistent", type=int, default=-1,
                   help="wide kernel under 'auto': 1 persistent grid, 0 one tile per cluster, -1 by K")
    args = p.parse_args()
    device = torch.device(args.device)
    from torch_einshard_b200.ops import _native, gemm
    mod = _native.require()
    writer = Writer(args.output)
    for name in args.shapes.split(","):
        m, n, k, a_mn, b_mn = SHAPES[name]
        a, b = make_operands(m, n, k, a_mn, b_mn, device)
        flops = 2.0 * m * n * k
        for kern in args.kernels.split(","):
            if kern == "cublas":
                fn = lambda: torch.matmul(a, b)  # noqa: E731
            else:
                mod.set_gemm_pair_mode({"1sm": 0, "2sm": 1, "wide": 2, "widep": 2, "streamk": -1, "auto": -1}[kern])
                mod.set_gemm_group_m(args.group_m)
                mod.set_gemm_split(args.split)
                mod.set_gemm_sleep_ns(args.sleep_ns)
                mod.set_tma_l2_promotion(args.l2_promotion)
                mod.set_gemm_persistent({"widep": 1, "wide": 0}.get(kern, args.persistent))
                mod.set_gemm_streamk({"streamk": 1, "auto": -1}.get(kern, 0))
                fn = lambda: gemm.native_bmm(a, b)  # noqa: E731
            label = f"gemm_{name}_{kern}"
            if args.mode == "burst":
                benchmark(label, fn, args=args, device=device, writer=writer, flops=flops,
                          extra={"M": m, "N": n, "K": k, "a_mn": a_mn, "b_mn": b_mn, "kernel": kern})
            else:
                ms, mhz, watts = sustained(fn, args.seconds)
                tflops = flops / (ms / 1e3) / 1e12
                writer.write({"name": label, "mode": "sustained", "ms": ms, "tflops": tflops,
                              "roofline_frac": tflops / peaks()["bf16_tflops_sustained"],
                              "roofline_of": "bf16_tflops_sustained", "sm_mhz_median": mhz,
                              "power_w_median": watts,
                              "tflops_per_ghz": tflops / (mhz / 1e3) if mhz else None,
                              "M": m, "N": n, "K": k, "a_mn": a_mn, "b_mn": b_mn, "kernel": kern})
        mod.set_gemm_pair_mode(-1)
        mod.set_gemm_group_m(0)
        mod.set_gemm_split(0)
        mod.set_gemm_persistent(-1)
        mod.set_gemm_streamk(-1)
        del a, b
        torch.cuda.empty_cache()
    _native.check_errors()


if __name__ == "__main__":
    main()
