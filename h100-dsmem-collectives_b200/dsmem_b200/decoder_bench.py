"""Timing of the Llama-2-7B decoder layer, one decode step, on one GPU.

    python -m dsmem_b200.decoder_bench            (from the package directory, or with it on PYTHONPATH)

hidden 4096, 32 heads x 128, FFN 11008 SwiGLU, eps 1e-5, RoPE theta 10000 at position S; bf16 weights
N(0, 0.02); bf16 KV caches of S = 4096 tokens N(0, 1), one per sequence; batch 1, 4, 16; cluster 4 and 8.
The step (seven launches) is captured in a CUDA graph of `reps` steps; the figure is the median over
rounds of the mean step time, CUDA events on the replay stream. Weights (405 MB) and caches exceed the
126 MB L2, so every step streams them from HBM. HBM roofline: bytes per step = weights
2 (4 h^2 + 3 ffn h) + per sequence 2 * 2 * S * h (K and V read) (+ activations, negligible);
frac = (bytes / time) / the measured HBM copy peak. `torch_unfused` times the same layer written with
torch.nn.functional (cuBLAS GEMMs, scaled_dot_product_attention) for comparison.
"""
from __future__ import annotations

import json
import math
import pathlib
import statistics

HID, HEADS, FFN, S = 4096, 32, 11008, 4096


def hbm_peak():
    p = pathlib.Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text()).get("hbm_gbs", 6650.0))
    return 6650.0


def _graph_time(fn, reps=10, rounds=5, warmup=3):
    import torch

    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(reps):
            fn()
    torch.cuda.synchronize()
    vals = []
    for _ in range(rounds):
        with torch.cuda.stream(stream):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
        torch.cuda.synchronize()
        vals.append(e0.elapsed_time(e1) * 1e3 / reps)
    del graph
    return statistics.median(vals)


def run(batches=(1, 4, 16), clusters=(4, 8), with_torch=True):
    import torch
    import torch.nn.functional as F

    from . import decoder_check, decoder_layer, rmsnorm_check

    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    bf = torch.bfloat16
    nrm = lambda *s, std=0.02, mean=0.0: (mean + std * torch.randn(*s, device=dev, generator=g)).to(bf)   # noqa: E731
    W = {"wqkv": nrm(3 * HID, HID), "wo": nrm(HID, HID), "wgu": nrm(2 * FFN, HID), "wd": nrm(HID, FFN),
         "w_rms": nrm(HID, std=0.02, mean=1.0), "w_post": nrm(HID, std=0.02, mean=1.0)}
    inv = 10000.0 ** (-torch.arange(0, 128, 2, dtype=torch.float64) / 128)
    ang = S * inv
    cos = torch.cat([ang.cos(), ang.cos()]).float().to(dev)
    sin = torch.cat([ang.sin(), ang.sin()]).float().to(dev)
    peak = hbm_peak()
    wbytes = 2 * (4 * HID * HID + 3 * FFN * HID)
    res = {"config": {"hidden": HID, "heads": HEADS, "head_dim": 128, "ffn": FFN, "seq_len": S, "dtype": "bf16",
                      "weights_bytes": wbytes, "hbm_peak_GBps": peak}, "batch": {}}
    for B in batches:
        cap = S + 1
        kc = nrm(B, cap, HEADS, 128, std=1.0)
        vc = nrm(B, cap, HEADS, 128, std=1.0)
        inp, rs = nrm(B, HID, std=1.0), nrm(B, HID, std=1.0)
        out, h = torch.empty_like(inp), torch.empty_like(inp)
        ws = torch.empty(1 << 22, dtype=torch.uint8, device=dev)
        bytes_step = wbytes + B * 2 * 2 * S * HID
        row = {}
        for n in clusters:
            def step(n=n):
                decoder_layer(inp, rs, W["w_rms"], W["wqkv"], W["wo"], W["w_post"], W["wgu"], W["wd"], kc, vc, cos,
                              sin, S, eps=1e-5, cluster_size=n, out=out, h_out=h, workspace=ws)
            us = _graph_time(step)
            decoder_check()
            rmsnorm_check()
            row[f"cluster{n}"] = {"us": round(us, 2), "tokens_per_s": round(B / (us * 1e-6), 1),
                                  "hbm_GBps": round(bytes_step / (us * 1e-6) / 1e9, 1),
                                  "hbm_frac": round(bytes_step / (us * 1e-6) / 1e9 / peak, 4)}
        if with_torch:
            K, V = kc[:, :S].float(), vc[:, :S].float()   # noqa: F841 - kept out of the timed step

            def torch_step():
                x = inp + rs
                xn = F.rms_norm(x, (HID,), W["w_rms"], 1e-5)
                qkv = F.linear(xn, W["wqkv"]).view(B, 3, HEADS, 128)
                q, k, v = qkv[:, 0], qkv[:, 1], qkv[:, 2]
                rot = lambda z: z * cos.to(bf) + torch.cat([-z[..., 64:], z[..., :64]], -1) * sin.to(bf)   # noqa: E731
                q, k = rot(q), rot(k)
                kc[:, S] = k
                vc[:, S] = v
                a = F.scaled_dot_product_attention(q.unsqueeze(2), kc.transpose(1, 2), vc.transpose(1, 2))
                o = F.linear(a.reshape(B, HID), W["wo"])
                hh = x + o
                hn = F.rms_norm(hh, (HID,), W["w_post"], 1e-5)
                gu = F.linear(hn, W["wgu"])
                return F.linear(F.silu(gu[:, :FFN]) * gu[:, FFN:], W["wd"])

            us = _graph_time(torch_step)
            row["torch_unfused"] = {"us": round(us, 2), "tokens_per_s": round(B / (us * 1e-6), 1),
                                    "hbm_GBps": round(bytes_step / (us * 1e-6) / 1e9, 1),
                                    "hbm_frac": round(bytes_step / (us * 1e-6) / 1e9 / peak, 4)}
        row["bytes_per_step"] = bytes_step
        res["batch"][str(B)] = row
        del kc, vc
        torch.cuda.empty_cache()
    return res


def main():
    import torch

    torch.cuda.set_device(0)
    print(json.dumps(run()), flush=True)


if __name__ == "__main__":
    main()
