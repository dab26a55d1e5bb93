#!/usr/bin/env python
"""Benchmark of the OSCAR INT2 rotated KV-cache hot path on B200.

One "step" is one OSCAR FULL-attention layer step of BASELINE config 3
(8 requests x 24576-token INT2 history, 4-token MTP, Hq 6 / Hk 1 / D 256,
128-token pages, sink 128 / recent 256 fp32 windows, clip 0.96 / 0.92):
rotate new K/V -> clip + INT2 store -> staging write -> rotate q -> paged
streaming attention -> output rotation.  Steps cycle over --layers
independent layers (their caches total > L2), so history is read from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl oscar|reference]

N > 1 runs under torchrun; every rank holds the same per-rank workload (one
tensor-parallel KV-head group, requests independent) -> weak scaling with no
data-path collective; the timed region is the max over ranks.
``--impl reference`` times the reference algorithm's CPU restatement (the
oracle) on the host cores for the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path
from types import SimpleNamespace as NS

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "INT2-KV attn query-tok/s & HBM GB/s vs peak; 8x24K MTP step latency"
UNIT = "query_tokens/s"
WORKLOAD = "cfg3_mtp_8x24k"
BYTES_PER_TOKEN_HEAD = 136  # 64 B K codes + 64 B V codes + 8 B scale/zero
BYTES_PER_STAGED = 2 * 256 * 4  # fp32 K and V staging rows of a staged (sink/recent) token


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["oscar", "reference"], default="oscar")
    ap.add_argument("--layers", type=int, default=12)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def workload_config(layers):
    from oscar_b200.synthetic import BASELINE_CONFIGS

    spec = BASELINE_CONFIGS[WORKLOAD]
    return dict(workload=WORKLOAD, requests=len(spec["prefixes"]), history_tokens=spec["prefixes"][0],
                mtp_tokens=spec["lengths"][0], hq=6, hk=1, head_dim=256, block_size=128, sink=128, recent=256,
                clip=[0.96, 0.92], layers_cycled=layers, global_batch=sum(spec["lengths"]),
                l2="inputs larger than L2: steps cycle over independent layers (>1 GB of caches)",
                parallelism="one TP KV-head group per GPU, replicated per rank (weak scaling)")


# ---------------------------------------------------------------------------
# GPU arm
def count_staged(torch, lay):
    """History positions whose staging seat is owned by their block (read from
    the fp32 staging rows instead of the INT2 codes)."""
    case = lay.case
    owner = lay.layer._oscar_slot_owner.reshape(-1)
    rows = owner.numel() // 128
    n = 0
    for r, (seq, ql) in enumerate(zip(case.seqs, np.diff(case.qsl))):
        pos = torch.arange(int(seq) - int(ql), device=owner.device)
        blk = case.bt[r, pos // 128].long()
        n += int((owner[(blk % rows) * 128 + pos % 128] == blk).sum())
    return n


def build_layers(torch, dev, n_layers):
    from oscar_b200 import synthetic
    from oscar_b200.backend import OscarAttentionBackendImpl

    spec = synthetic.BASELINE_CONFIGS[WORKLOAD]
    impl = OscarAttentionBackendImpl.create(6, 1, 256)
    cfg = impl._oscar
    cfg.sink_tokens, cfg.recent_tokens, cfg.staging_tokens = 128, 256, 8192
    cfg.k_clip_ratio, cfg.v_clip_ratio = 0.96, 0.92
    cfg.window_enabled = True
    layers = []
    for li in range(n_layers):
        case = synthetic.make_case(spec["prefixes"], spec["lengths"], hk=1, group=6, seed=1000 + li, device=dev)
        synthetic.fill_caches(case)
        g = torch.Generator(device=dev).manual_seed(7 + li)
        rk = torch.linalg.qr(torch.randn(256, 256, generator=g, device=dev)).Q.contiguous()
        rv = torch.linalg.qr(torch.randn(256, 256, generator=g, device=dev)).Q.contiguous()
        layer = NS(layer_name=f"model.layers.{li}.self_attn.attn", _oscar_rots=(rk, rv))
        cache = (case.kc, case.vc)
        impl._set_caches(cache)
        impl._ensure_staging(layer, cache)
        sk, sv, owner = case.stage
        layer._oscar_stage_k.copy_(sk)
        layer._oscar_stage_v.copy_(sv)
        layer._oscar_slot_owner.copy_(owner)
        slots = []
        for r, (p, n) in enumerate(zip(spec["prefixes"], spec["lengths"])):
            pos = torch.arange(p, p + n, device=dev)
            slots.append(case.bt[r, pos // 128].long() * 128 + pos % 128)
        md = NS(num_actual_tokens=case.q.shape[0], slot_mapping=torch.cat(slots), query_start_loc_cpu=torch.tensor(case.qsl),
                seq_lens_list=case.seqs, block_tables=case.bt,
                query_start_loc=torch.tensor(case.qsl, dtype=torch.int32, device=dev),
                seq_lens=torch.tensor(case.seqs, dtype=torch.int32, device=dev))
        out = torch.empty(case.q.shape[0], 6 * 256, dtype=torch.bfloat16, device=dev)
        # the step's inputs live in one device buffer (q, k, v views), as an engine's persistent
        # input buffers do, so that the end-to-end loop fills them with one host copy
        nq, nk, nv = case.q.numel(), case.k_new.numel(), case.v_new.numel()
        io = torch.empty(nq + nk + nv, dtype=torch.bfloat16, device=dev)
        q, k, v = io[:nq].view(case.q.shape), io[nq:nq + nk].view(case.k_new.shape), io[nq + nk:].view(case.v_new.shape)
        q.copy_(case.q)
        k.copy_(case.k_new)
        v.copy_(case.v_new)
        layers.append(NS(layer=layer, cache=cache, q=q, k=k, v=v, io=io, md=md, out=out, case=case))
        del case.old_k, case.old_v
    torch.cuda.synchronize(dev)
    return impl, layers


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"oscar_clocks_{os.getpid()}.csv"

    def start(self):
        """Start sampling and wait for the first sample, so that the sampler's
        start-up (driver initialisation) is over before any timed region."""
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.gpu)], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 10.0 and self.proc.poll() is None:
            if self.path.exists() and self.path.stat().st_size > 0:
                break
            time.sleep(0.05)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm), "reasons": sorted(reasons)}


def timed(torch, dev, fn, steps, dist, preroll=True):
    """Device time of `steps` calls (CUDA events), barrier + sync on both sides,
    max over ranks.  A spin kernel issued before the start event lets the host
    enqueue ahead so the region measures the device, not Python launch cost."""
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if preroll:
        torch.cuda._sleep(int(2_000_000 * max(1, steps)))
    start.record()
    for i in range(steps):
        fn(i)
    end.record()
    torch.cuda.synchronize(dev)
    ms = start.elapsed_time(end)
    if dist is not None:
        from oscar_b200.shards import max_over_ranks

        ms = max_over_ranks(ms, device=dev)
        dist.barrier()
    return ms


def cpu_baseline_sample(lay):
    """The oracle (reference algorithm restated on the CPU) on one request of
    the workload: clip+store of its 4 new tokens and its attention read."""
    import torch

    from oracle import oscar_oracle as orc

    c = lay.case
    k8 = c.kc.view(torch.uint8).cpu().numpy()
    v8 = c.vc.view(torch.uint8).cpu().numpy()
    stage = tuple(t.cpu().numpy() for t in (lay.layer._oscar_stage_k, lay.layer._oscar_stage_v, lay.layer._oscar_slot_owner))
    q = c.q[:4].float().cpu().numpy()
    kn = c.k_new[:4].float().cpu().numpy()
    vn = c.v_new[:4].float().cpu().numpy()
    rk, rv = (t.cpu().numpy() for t in lay.layer._oscar_rots)
    bt = c.bt[:1].cpu().numpy()
    slots = lay.md.slot_mapping[:4].cpu().numpy()
    reps, t0 = 0, time.perf_counter()
    while True:
        k8w, v8w = k8.copy(), v8.copy()
        orc.store(orc.rotate_clip(kn, rk, 0.96), orc.rotate_clip(vn, rv, 0.92), k8w, v8w, slots)
        qr = orc.round_bf16(q @ rk)
        orc.streaming_attention(qr, orc.round_bf16(kn @ rk), orc.round_bf16(vn @ rv), k8w, v8w, bt, [0, 4],
                                [c.seqs[0]], c.scale, stage)
        reps += 1
        if time.perf_counter() - t0 > 10.0 or reps >= 20:
            break
    dt = (time.perf_counter() - t0) / reps
    return {"value": 4.0 / dt, "unit": UNIT, "cores": 1, "kind": "port",
            "sample": f"1 of 8 requests (24576 history + 4 MTP tokens): rotate/clip/store + attention, "
                      f"numpy oracle, {reps} reps, {dt * 1e3:.1f} ms each"}


def run_gpu(args):
    import torch

    from oscar_b200 import _native, kernels
    from oscar_b200.graphs import GraphedForward, GraphedSequence

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    impl, layers = build_layers(torch, dev, args.layers)
    L = len(layers)
    lib = _native.lib()

    def step(i):
        lay = layers[i % L]
        impl.forward(lay.layer, lay.q, lay.k, lay.v, lay.cache, lay.md, output=lay.out)

    clocks = ClockSampler(dev.index)
    clocks.start()
    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize(dev)
    # bit-level sanity: no bounds violations in warm-up
    assert kernels.device_error(dev) == 0
    n0 = lib.oscar_launch_count()
    step(0)
    launches_per_step = lib.oscar_launch_count() - n0
    torch.cuda.synchronize(dev)

    # decode steps replay CUDA graphs (as vLLM does, which captures a whole model
    # forward): the timed region is ONE graph of exactly `steps` layer forwards,
    # cycling over the layers, so consecutive layers' kernels overlap the way
    # they do inside a model graph; warm-up replays a graph of `warmup` of them.
    # (Per-layer graphs, used for the end-to-end number below, add a graph launch
    # of a few microseconds between layers.)
    pool = torch.cuda.graph_pool_handle()
    graphs = [GraphedForward(impl, lay.layer, lay.q, lay.k, lay.v, lay.cache, lay.md, lay.out, pool=pool)
              for lay in layers]

    def seq(n):
        return GraphedSequence([(impl, layers[i % L].layer, layers[i % L].q, layers[i % L].k, layers[i % L].v,
                                 layers[i % L].cache, layers[i % L].md, layers[i % L].out) for i in range(n)],
                               pool=pool)

    warm_graph = seq(max(args.warmup, 3))
    timed_graph = seq(args.steps)
    warm_graph.replay()
    torch.cuda.synchronize(dev)
    assert kernels.device_error(dev) == 0
    ms = timed(torch, dev, lambda i: timed_graph.replay(), 1, dist)
    assert kernels.device_error(dev) == 0

    def graph_step(i):
        graphs[i % L].replay()

    ms_layer_graphs = timed(torch, dev, graph_step, args.steps, dist)
    launches = launches_per_step * args.steps
    ms_host_paced = timed(torch, dev, step, args.steps, dist, preroll=False)
    clk = clocks.stop()

    # attention pass alone (decode kernel + combine) for the roofline
    rot = []
    for lay in layers:
        rk, rv = lay.layer._oscar_rots
        n = lay.q.shape[0]
        qr = torch.matmul(lay.q.float().view(-1, 256), rk).view(n, 6, 256).bfloat16()
        kr = torch.matmul(lay.k.float().view(-1, 256), rk).view(n, 1, 256).bfloat16()
        vr = torch.matmul(lay.v.float().view(-1, 256), rv).view(n, 1, 256).bfloat16()
        stage = (lay.layer._oscar_stage_k, lay.layer._oscar_stage_v, lay.layer._oscar_slot_owner)
        rot.append((qr, kr, vr, lay.cache[0], lay.cache[1], lay.md.block_tables, lay.case.qsl, lay.case.seqs,
                    lay.case.scale, stage))

    def attn(i):
        kernels.slab_attention(*rot[i % L])

    for i in range(3):
        attn(i)
    n_attn = max(args.steps, 2 * L)
    ms_attn = timed(torch, dev, attn, n_attn, dist) / n_attn
    hist = sum(layers[0].case.seqs) - layers[0].q.shape[0]
    staged = count_staged(torch, layers[0])
    alg_bytes = BYTES_PER_TOKEN_HEAD * hist + BYTES_PER_STAGED * staged
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(peaks.get("hbm_gbs", 6650.0))
    achieved = alg_bytes / (ms_attn * 1e-3) / 1e9
    traffic = None
    tf = ROOT / "profiles" / "attention_traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get("bytes_per_launch")

    # end to end through the backend with host buffers (pinned in, pinned out)
    lay0 = layers[0]
    hio_b = [lay.io.cpu().pin_memory() for lay in layers]  # q, k, v of the step, packed
    ho_b = [torch.empty(lay.out.shape, dtype=lay.out.dtype).pin_memory() for lay in layers]

    def e2e_step(i):
        # host inputs (one pinned buffer: q, k, v) into the graph's static tensors, replay,
        # result back to the host
        j = i % L
        lay = layers[j]
        lay.io.copy_(hio_b[j], non_blocking=True)
        graphs[j].replay()
        ho_b[j].copy_(lay.out, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()

    for i in range(3):
        e2e_step(i)
    ms_e2e = timed(torch, dev, e2e_step, args.steps, dist, preroll=False)
    h2d = hio_b[0].numel() * 2
    d2h = ho_b[0].numel() * 2

    tokens = lay0.q.shape[0]
    ms_step = ms / args.steps
    result = {
        "metric": METRIC, "value": world * tokens / (ms_step * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(L),
        "step_latency_us": ms_step * 1e3,
        "ms_per_step_eager_host_paced": ms_host_paced / args.steps,
        "step_mode": "one CUDA graph of the timed steps' layer forwards (oscar_b200.graphs.GraphedSequence), "
                     "replayed once",
        "ms_per_step_graph_per_layer": ms_layer_graphs / args.steps,
        "e2e": {"value": world * tokens / (ms_e2e / args.steps * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": ms_e2e / args.steps},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "kernel": "slab attention pass (decode_tc_kernel + tc_combine_kernel)",
                     "launch_us": ms_attn * 1e3, "algorithmic_bytes": alg_bytes, "staged_tokens": staged,
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if peaks else "fallback 6650 GB/s"},
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            result["cpu_baseline"] = cpu_baseline_sample(layers[0])
        except Exception as exc:  # keep the bench line even if the sample fails
            result["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": 1, "kind": "port", "sample": f"failed: {exc}"}
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


# ---------------------------------------------------------------------------
# reference arm: the oracle on the host cores
_REF = {}


def _ref_attend(req):
    from oracle import oscar_oracle as orc

    d = _REF
    a, b = d["qsl"][req], d["qsl"][req + 1]
    out, _ = orc.streaming_attention(d["qr"][a:b], d["kr"][a:b], d["vr"][a:b], d["k8"], d["v8"], d["bt"][req:req + 1],
                                     [0, b - a], [d["seqs"][req]], d["scale"], d["stage"])
    return out


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import multiprocessing as mp

    import torch

    from oracle import oscar_oracle as orc
    from oscar_b200 import synthetic

    spec = synthetic.BASELINE_CONFIGS[WORKLOAD]
    case = synthetic.make_case(spec["prefixes"], spec["lengths"], hk=1, group=6, seed=1000)
    k8 = case.kc.view(torch.uint8).numpy().copy()
    v8 = case.vc.view(torch.uint8).numpy().copy()
    orc.store(case.old_k.numpy(), case.old_v.numpy(), k8, v8, case.slots.numpy())
    g = torch.Generator().manual_seed(7)
    rk = torch.linalg.qr(torch.randn(256, 256, generator=g)).Q.numpy().astype(np.float32)
    rv = torch.linalg.qr(torch.randn(256, 256, generator=g)).Q.numpy().astype(np.float32)
    st = orc.Staging(128, 1, 256, 128, 256, 8192)
    sk, sv, owner = (t.numpy() for t in case.stage)
    st.stage_k[:], st.stage_v[:], st.owner[:] = sk, sv, owner
    q = case.q.float().numpy()
    kn = case.k_new.float().numpy()
    vn = case.v_new.float().numpy()
    slots = []
    for r, (p, n) in enumerate(zip(spec["prefixes"], spec["lengths"])):
        pos = np.arange(p, p + n)
        slots.append(case.bt[r].numpy()[pos // 128].astype(np.int64) * 128 + pos % 128)
    slots = np.concatenate(slots)
    cores = os.cpu_count() or 1
    nproc = max(1, min(cores, len(spec["prefixes"])))

    def host_write():
        kr_unclipped, vr_unclipped = kn @ rk, vn @ rv
        orc.store(orc.clip_only(kr_unclipped, 0.96), orc.clip_only(vr_unclipped, 0.92), k8, v8, slots)
        st.write(kn, vn, rk, rv, slots, case.qsl, case.seqs, len(slots))
        return orc.round_bf16(q @ rk), orc.round_bf16(kr_unclipped), orc.round_bf16(vr_unclipped)

    # One write before forking: the workers inherit the written caches/staging,
    # and every later step writes the same bytes again (the MTP slots repeat).
    qr, kr, vr = host_write()
    _REF.update(k8=k8, v8=v8, bt=case.bt.numpy(), qsl=case.qsl, seqs=case.seqs, scale=case.scale, stage=st.tuple(),
                qr=qr, kr=kr, vr=vr)
    ctx = mp.get_context("fork")  # this arm never initialises CUDA

    def one_step(pool):
        host_write()
        outs = pool.map(_ref_attend, range(len(spec["prefixes"])))
        return np.concatenate(outs) @ rv.T

    with ctx.Pool(nproc) as pool:
        for _ in range(args.warmup):
            one_step(pool)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            one_step(pool)
        dt = (time.perf_counter() - t0) / args.steps
    tokens = sum(spec["lengths"])
    value = tokens / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": workload_config(1),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": nproc, "kind": "port",
                         "sample": "full cfg3 layer step (8 x 24576 history + 4 MTP tokens) on the numpy oracle, "
                                   f"requests spread over {nproc} forked processes"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
