"""Small, self-contained workloads for Nsight Compute captures (python -m dsmem_b200.profile --case ...).

Each case allocates its inputs, runs `--warmup` untimed launches and then `--launches` launches of one
kernel, and exits; sized so a full-section capture of one to three launches ends in a minute or two
(inputs above the 126 MB L2, a few hundred MB on the device at most).
  allreduce   batch AllReduce through the C ABI (--alg, --cluster, --payload, --problems, --dtype)
  rmsnorm     cluster-fused RMSNorm (--rows, --hidden, --cluster)
  decoder     one Llama-2-7B decoder-layer step (--batch, --cluster; 4096 cached tokens): its seven launches
  rowwise     a row-wise reduction-reuse kernel (--workload, --rows, --cols, --cluster; fp32, 5 + cols rows seed)
  topk        exact top-k (--rows, --cols as the row length n, --k, --cluster; randn rows)
"""
import argparse
import pathlib
import sys

PKG = pathlib.Path(__file__).resolve().parent.parent
if str(PKG) not in sys.path:
    sys.path.insert(0, str(PKG))

import dsmem_b200 as D  # noqa: E402


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", choices=["allreduce", "rmsnorm", "decoder", "rowwise", "topk"], default="allreduce")
    ap.add_argument("--k", type=int, default=2048)
    ap.add_argument("--workload", default="lars_momentum")
    ap.add_argument("--cols", type=int, default=16384)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--alg", default="two_shot_push")
    ap.add_argument("--cluster", type=int, default=8)
    ap.add_argument("--payload", type=int, default=65536)
    ap.add_argument("--problems", type=int, default=512)
    ap.add_argument("--dtype", choices=["f32", "bf16", "i32"], default="f32")
    ap.add_argument("--rows", type=int, default=4096)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--no-pipeline", action="store_true")
    args = ap.parse_args(argv)
    import torch

    torch.cuda.set_device(0)
    if args.case == "allreduce":
        dt = {"f32": D.Dtype.F32, "bf16": D.Dtype.BF16, "i32": D.Dtype.I32}[args.dtype]
        tdt = {D.Dtype.F32: torch.float32, D.Dtype.BF16: torch.bfloat16, D.Dtype.I32: torch.int32}[dt]
        n, p = args.cluster, args.payload
        m = D.msg_elems(D.Op.ALLREDUCE, n, p, dt)
        count = args.problems * n * m
        tin = (torch.rand(count, device="cuda") * 2 - 1).to(tdt) if dt != D.Dtype.I32 else \
            torch.randint(-1000, 1000, (count,), dtype=torch.int32, device="cuda")
        tout = torch.empty_like(tin)
        alg = D.Alg[args.alg.upper()]
        D.set_pipelined(not args.no_pipeline)
        for _ in range(args.warmup + args.launches):
            D.collective(D.Op.ALLREDUCE, alg, tin, tout, n, p)
        D.check()
    elif args.case == "rowwise":
        from dsmem_b200 import rowwise_bench as RB

        gen = torch.Generator(device="cuda")
        gen.manual_seed(5 + args.cols)
        ins, outs = RB.make_set(torch, args.workload, args.rows, args.cols, gen)
        for _ in range(args.warmup + args.launches):
            RB.launch(args.workload, ins, outs, args.cluster)
        torch.cuda.synchronize()
        D.rowwise_check()
    elif args.case == "topk":
        gen = torch.Generator(device="cuda")
        gen.manual_seed(args.rows * args.cols)
        x = torch.randn(args.rows, args.cols, device="cuda", generator=gen)
        out = torch.empty(args.rows, args.k, dtype=torch.int32, device="cuda")
        for _ in range(args.warmup + args.launches):
            D.topk(x, k=args.k, cluster_size=args.cluster, out=out)
        torch.cuda.synchronize()
        D.topk_check()
    elif args.case == "decoder":
        hid, heads, ffn, S, B = 4096, 32, 11008, 4096, args.batch
        nrm = lambda *s, std=0.02, mean=0.0: (mean + std * torch.randn(*s, device="cuda")).to(torch.bfloat16)  # noqa: E731
        w = [nrm(hid, mean=1.0), nrm(3 * hid, hid), nrm(hid, hid), nrm(hid, mean=1.0), nrm(2 * ffn, hid), nrm(hid, ffn)]
        kc, vc = nrm(B, S + 1, heads, 128, std=1.0), nrm(B, S + 1, heads, 128, std=1.0)
        inp, res = nrm(B, hid, std=1.0), nrm(B, hid, std=1.0)
        cos, sin = torch.ones(128, device="cuda"), torch.zeros(128, device="cuda")
        for _ in range(args.warmup + args.launches):
            D.decoder_layer(inp, res, *w, kc, vc, cos, sin, S, eps=1e-5, cluster_size=args.cluster)
        torch.cuda.synchronize()
        D.decoder_check()
    else:
        x = torch.randn(args.rows, args.hidden, device="cuda").to(torch.bfloat16)
        w = (1 + 0.02 * torch.randn(args.hidden, device="cuda")).to(torch.bfloat16)
        y = torch.empty_like(x)
        for _ in range(args.warmup + args.launches):
            D.rmsnorm(x, w, 1e-6, cluster_size=args.cluster, out=y)
        torch.cuda.synchronize()
        D.rmsnorm_check()
    torch.cuda.synchronize()
    print("profile case done", args.case)


if __name__ == "__main__":
    main()
