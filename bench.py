#!/usr/bin/env python
"""Benchmark of the OSCAR INT2 rotated KV-cache hot path on B200.

Headline: one OSCAR FULL-attention layer step of BASELINE config 3 for the
whole model layer (8 requests x 24576-token INT2 history, 4-token MTP, Hq 24 /
Hk 4 = four KV-head groups of Hq 6 / Hk 1, D 256, 128-token pages, sink 128 /
recent 256 fp32 windows, clip 0.96 / 0.92, QR rotations): rotate new K/V ->
clip + INT2 store -> staging write -> rotate q -> paged streaming attention ->
output rotation.  Steps cycle over --layers independent layers (their caches
total > L2), so history is read from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl oscar|reference]

One fixed global workload, strongly scaled over N ranks (one per GPU, launched
by torchrun): the four KV-head groups are divided among the ranks (4 on 1 GPU,
2 each on 2, 1 each on 4); on 8 GPUs each rank takes one group and half of the
requests.  Outputs of different ranks are disjoint (vLLM's tensor-parallel
layout), so this step needs no collective.  Secondary lines in the same JSON:

* ``cfg3_split_kv`` (8 ranks): the same step with each request's history cut
  into two page-aligned shards held by the two ranks of a KV-head group; the
  pair exchanges its partial (O, LSE) by NCCL all-gather and folds them with
  merge_slab, inside the timed region, checked against the rank's own
  single-pass result;
* ``cfg4_continuation``: 15360 new tokens on 9256 tokens of history, split by
  KV-head group up to 4 ranks and, on 8, by query heads (3 of a group's 6 per
  rank, the KV head replicated as vLLM does at tensor-parallel 8);
* ``cfg5_mixed_16l``: 64 mixed requests, 16 layers, MTP-reject rewrites,
  split like the headline (on 8 ranks, request halves of equal history).

``--impl reference`` times the reference algorithm's CPU restatement (the
oracle) on the host cores.
"""
from __future__ import annotations

import argparse
import json
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
GROUPS = 4          # KV-head groups of the model layer (Hk 4)
GROUP_HQ = 6        # query heads per group
D = 256
BYTES_PER_TOKEN_HEAD = 136  # 64 B K codes + 64 B V codes + 8 B scale/zero
BYTES_PER_STAGED = 2 * D * 4  # fp32 K and V staging rows of a staged (sink/recent) token


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["oscar", "reference"], default="oscar")
    ap.add_argument("--layers", type=int, default=6)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="skip the cfg4 / cfg5 measurements")
    ap.add_argument("--only", choices=["cfg4", "cfg5", "split_kv"], default=None,
                    help="run one secondary workload alone and print its JSON object (profiling)")
    ap.add_argument("--workspace-mib", type=int, default=None,
                    help="attention workspace bound of the backend (default: the OSCAR_ASCEND_STREAM_WORKSPACE_MIB "
                         "default, 128)")
    return ap.parse_args()


def shard_plan(world: int, rank: int, n_requests: int) -> NS:
    """This rank's share of the global workload: KV-head groups [g0, g1) and
    requests [r0, r1); on more ranks than groups, the ranks of a group split its
    requests (headline, cfg5), its history (cfg3 split-KV) or its query heads
    (cfg4); this rank is part ``split`` of ``splits``."""
    if world <= GROUPS:
        per = GROUPS // world
        if per * world != GROUPS:
            raise SystemExit(f"--gpus {world}: the {GROUPS} KV-head groups must divide evenly")
        g0 = rank * per
        return NS(g0=g0, g1=g0 + per, r0=0, r1=n_requests, split=0, splits=1, pair=None)
    if world % GROUPS:
        raise SystemExit(f"--gpus {world}: a multiple of {GROUPS} is needed beyond {GROUPS} ranks")
    share = world // GROUPS
    g = rank // share
    part = rank % share
    per_req = -(-n_requests // share)
    r0, r1 = min(n_requests, part * per_req), min(n_requests, (part + 1) * per_req)
    return NS(g0=g, g1=g + 1, r0=r0, r1=r1, split=part, splits=share,
              pair=[g * share + i for i in range(share)])


def workload_config(layers, plan, world):
    return dict(workload=WORKLOAD, requests=8, history_tokens=24576, mtp_tokens=4, hq=GROUPS * GROUP_HQ, hk=GROUPS,
                head_dim=D, block_size=128, sink=128, recent=256, clip=[0.96, 0.92], layers_cycled=layers,
                global_batch=32, l2="inputs larger than L2: steps cycle over independent layers (>1 GB of caches)",
                parallelism=(f"{world} rank(s): KV-head groups split over ranks; rank 0 holds groups "
                             f"[{plan.g0}, {plan.g1}) and requests [{plan.r0}, {plan.r1})"))


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




# ---------------------------------------------------------------------------
# GPU arm
def slice_case(torch, case, g0, g1, r0, r1, group=GROUP_HQ):
    """The part of a full-model case (Hk = GROUPS) that one rank serves: KV-head
    groups [g0, g1) (their query heads) and requests [r0, r1)."""
    qsl = case.qsl
    tok0, tok1 = qsl[r0], qsl[r1]
    sk, sv, owner = case.stage
    return NS(q=case.q[tok0:tok1, group * g0:group * g1].contiguous(),
              k_new=case.k_new[tok0:tok1, g0:g1].contiguous(), v_new=case.v_new[tok0:tok1, g0:g1].contiguous(),
              kc=case.kc[:, :, g0:g1].contiguous(), vc=case.vc[:, :, g0:g1].contiguous(),
              bt=case.bt[r0:r1].contiguous(), qsl=[x - tok0 for x in qsl[r0:r1 + 1]], seqs=list(case.seqs[r0:r1]),
              scale=case.scale, stage=(sk[:, :, g0:g1].contiguous(), sv[:, :, g0:g1].contiguous(), owner.clone()))


def qr_pair(torch, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    rk = torch.linalg.qr(torch.randn(D, D, generator=g, device=dev)).Q.contiguous()
    rv = torch.linalg.qr(torch.randn(D, D, generator=g, device=dev)).Q.contiguous()
    return rk, rv


BACKEND_ENV = {"OSCAR_ASCEND_SINK_TOKENS": "128", "OSCAR_ASCEND_RECENT_TOKENS": "256",
               "OSCAR_ASCEND_STAGING_TOKENS": "8192", "OSCAR_ASCEND_K_CLIP_RATIO": "0.96",
               "OSCAR_ASCEND_V_CLIP_RATIO": "0.92", "OSCAR_ASCEND_ATTENTION_MODE": "streaming",
               "OSCAR_ASCEND_VERBOSE": "0"}


def make_backend(hk, args, hq=None):
    """The backend impl, configured through its environment keys; the
    effective configuration goes to stderr (the rotations are seeded QR
    matrices attached to each layer, not a checkpoint path)."""
    from oscar_b200.backend import OscarAttentionBackendImpl

    os.environ.update(BACKEND_ENV)
    if args.workspace_mib is not None:
        os.environ["OSCAR_ASCEND_STREAM_WORKSPACE_MIB"] = str(args.workspace_mib)
    impl = OscarAttentionBackendImpl.create(hq or GROUP_HQ * hk, hk, D)
    cfg = impl._oscar
    print(f"[bench] OSCAR backend: Hq={impl.num_heads} Hk={impl.num_kv_heads} D={D} sink={cfg.sink_tokens} "
          f"recent={cfg.recent_tokens} staging={cfg.staging_tokens} clip={cfg.k_clip_ratio}/{cfg.v_clip_ratio} "
          f"mode={cfg.attention_mode} workspace={cfg.stream_workspace_bytes >> 20} MiB rotations=seeded QR per layer",
          file=sys.stderr, flush=True)
    return impl


def build_layers(torch, dev, n_layers, plan, args):
    """The rank's share of --layers independent cfg3 layers (seeded per layer,
    identical on every rank before slicing)."""
    from oscar_b200 import synthetic

    prefixes, lengths = [24576] * 8, [4] * 8
    hk = plan.g1 - plan.g0
    impl = make_backend(hk, args)
    layers = []
    for li in range(n_layers):
        full = synthetic.make_case(prefixes, lengths, hk=GROUPS, group=GROUP_HQ, seed=1000 + li, device=dev)
        synthetic.fill_caches(full)
        del full.old_k, full.old_v
        case = slice_case(torch, full, plan.g0, plan.g1, plan.r0, plan.r1)
        del full
        rk, rv = qr_pair(torch, 7 + li, dev)
        layer = NS(layer_name=f"model.layers.{li}.self_attn.attn", _oscar_rots=(rk, rv))
        cache = (case.kc, case.vc)
        impl._set_caches(cache)
        impl._ensure_staging(layer, cache)
        for dst, src in zip((layer._oscar_stage_k, layer._oscar_stage_v, layer._oscar_slot_owner), case.stage):
            dst.copy_(src)
        slots = []
        for r in range(plan.r1 - plan.r0):
            pos = torch.arange(prefixes[0], prefixes[0] + lengths[0], device=dev)
            slots.append(case.bt[r, pos // 128].long() * 128 + pos % 128)
        n = case.q.shape[0]
        md = NS(num_actual_tokens=n, slot_mapping=torch.cat(slots), query_start_loc_cpu=torch.tensor(case.qsl),
                seq_lens_list=case.seqs, block_tables=case.bt,
                query_start_loc=torch.tensor(case.qsl, dtype=torch.int32, device=dev),
                seq_lens=torch.tensor(case.seqs, dtype=torch.int32, device=dev))
        out = torch.empty(n, GROUP_HQ * hk * D, dtype=torch.bfloat16, device=dev)
        # the step's inputs live in one device buffer (q, k, v views), as an engine's persistent
        # input buffers do, so that the end-to-end loop fills them with one host copy
        nq, nk = case.q.numel(), case.k_new.numel()
        io = torch.empty(nq + 2 * nk, dtype=torch.bfloat16, device=dev)
        q, k, v = io[:nq].view(case.q.shape), io[nq:nq + nk].view(case.k_new.shape), io[nq + nk:].view(case.v_new.shape)
        q.copy_(case.q)
        k.copy_(case.k_new)
        v.copy_(case.v_new)
        layers.append(NS(layer=layer, cache=cache, q=q, k=k, v=v, io=io, md=md, out=out, case=case))
    torch.cuda.synchronize(dev)
    return impl, layers


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


def cpu_baseline_sample(lay, plan):
    """The oracle (the reference algorithm restated on the CPU) on one of the
    workload's 32 (request, KV-head group) units: clip + store of its 4 new
    tokens and its attention read, on one core; the full step is 32 such units."""
    import torch

    from oracle import oscar_oracle as orc

    c = lay.case
    k8 = c.kc.view(torch.uint8)[:, :, 0:1].cpu().numpy().copy()
    v8 = c.vc.view(torch.uint8)[:, :, 0:1].cpu().numpy().copy()
    sk, sv, owner = (lay.layer._oscar_stage_k, lay.layer._oscar_stage_v, lay.layer._oscar_slot_owner)
    stage = (sk[:, :, 0:1].cpu().numpy(), sv[:, :, 0:1].cpu().numpy(), owner.cpu().numpy())
    q = c.q[:4, :GROUP_HQ].float().cpu().numpy()
    kn = c.k_new[:4, 0:1].float().cpu().numpy()
    vn = c.v_new[:4, 0:1].float().cpu().numpy()
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
    units = 8 * GROUPS
    return {"value": 32.0 / (dt * units), "unit": UNIT, "cores": 1, "kind": "port",
            "sample": f"1 of the step's {units} (request, KV-head group) units (24576 history + 4 MTP tokens, "
                      f"Hq 6 / Hk 1): rotate/clip/store + attention on the numpy oracle, {reps} reps of "
                      f"{dt * 1e3:.1f} ms; value = 32 query tokens / ({units} x that time)"}


def load_peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    peaks = json.loads(f.read_text()) if f.exists() else {}
    src = "MEASURED_PEAKS.json (of measured)" if peaks else "fallback (of fallback)"
    return (float(peaks.get("hbm_gbs", 6650.0)), float(peaks.get("bf16_tflops", 1590.0)),
            float(peaks.get("bf16_tflops_sustained", 1400.0)), src)


def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    return world, rank, dist, dev


def pair_groups(dist, world):
    """NCCL groups of the ranks that share one KV-head group (8 ranks: pairs);
    every rank creates every group, in the same order."""
    if dist is None or world <= GROUPS:
        return None
    share = world // GROUPS
    mine = None
    for g in range(GROUPS):
        ranks = [g * share + i for i in range(share)]
        grp = dist.new_group(ranks)
        if dist.get_rank() in ranks:
            mine = grp
    return mine


# ---------------------------------------------------------------------------
# headline: the cfg3 model-layer step
def run_headline(torch, dev, args, world, rank, dist, plan):
    from oscar_b200 import _native, kernels
    from oscar_b200.graphs import GraphedForward, GraphedSequence

    impl, layers = build_layers(torch, dev, args.layers, plan, args)
    L = len(layers)
    lib = _native.lib()

    def step(i):
        lay = layers[i % L]
        impl.forward(lay.layer, lay.q, lay.k, lay.v, lay.cache, lay.md, output=lay.out)

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize(dev)
    assert kernels.device_error(dev) == 0
    n0 = lib.oscar_launch_count()
    step(0)
    launches_per_step = lib.oscar_launch_count() - n0
    torch.cuda.synchronize(dev)

    # Decode steps replay CUDA graphs, as vLLM does (it captures a whole model
    # forward): the timed region is ONE graph of exactly `steps` layer forwards
    # cycling over the layers, so consecutive layers' kernels overlap as inside
    # a model graph.  Per-layer graphs (used end to end) add a graph launch
    # between layers; the eager figure is the host-paced backend API.
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
    clocks = ClockSampler(dev.index)
    clocks.start()
    ms = timed(torch, dev, lambda i: timed_graph.replay(), 1, dist)
    clk = clocks.stop()
    assert kernels.device_error(dev) == 0
    ms_layer_graphs = timed(torch, dev, lambda i: graphs[i % L].replay(), args.steps, dist)
    ms_host_paced = timed(torch, dev, step, args.steps, dist, preroll=False)

    # the attention pass alone (decode kernel + combine) on the step's rotated inputs: the roofline
    rot = []
    for lay in layers:
        rk, rv = lay.layer._oscar_rots
        n = lay.q.shape[0]
        hq = lay.q.numel() // (n * D)
        hk = lay.k.shape[1]
        qr = torch.matmul(lay.q.float().view(-1, D), rk).view(n, hq, D).bfloat16()
        kr = torch.matmul(lay.k.float().view(-1, D), rk).view(n, hk, D).bfloat16()
        vr = torch.matmul(lay.v.float().view(-1, D), rv).view(n, hk, D).bfloat16()
        stage = (lay.layer._oscar_stage_k, lay.layer._oscar_stage_v, lay.layer._oscar_slot_owner)
        rot.append((qr, kr, vr, lay.cache[0], lay.cache[1], lay.md.block_tables, lay.case.qsl, lay.case.seqs,
                    lay.case.scale, stage))

    def attn(i):
        kernels.slab_attention(*rot[i % L])

    for i in range(3):
        attn(i)
    n_attn = max(args.steps, 2 * L)
    ms_attn = timed(torch, dev, attn, n_attn, dist) / n_attn
    hk = plan.g1 - plan.g0
    hist = sum(layers[0].case.seqs) - layers[0].q.shape[0]
    staged = count_staged(torch, layers[0])
    alg_bytes = hk * (BYTES_PER_TOKEN_HEAD * hist + BYTES_PER_STAGED * staged)

    # end to end through the backend with host buffers, as an engine pipelines
    # steps: every step copies its q/k/v (one pinned buffer) in on one copy
    # stream -- overlapping the step in front -- replays its layer's graph once
    # they have landed, and copies the output back to pinned host memory on a
    # second copy stream once the replay is done; the host waits once, at the end
    main = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)   # host -> device
    back = torch.cuda.Stream(dev)   # device -> host
    hio_b = [lay.io.cpu().pin_memory() for lay in layers]
    ho_b = [torch.empty(lay.out.shape, dtype=lay.out.dtype).pin_memory() for lay in layers]
    ev_in = [torch.cuda.Event() for _ in layers]
    ev_done = [torch.cuda.Event() for _ in layers]
    ev_out = [torch.cuda.Event() for _ in layers]
    for j in range(L):  # created and complete before the first wait
        for ev in (ev_in[j], ev_done[j], ev_out[j]):
            ev.record(main)

    def e2e_step(i):
        j = i % L
        lay = layers[j]
        copy.wait_event(ev_done[j])  # the previous replay of this layer has read its inputs
        with torch.cuda.stream(copy):
            lay.io.copy_(hio_b[j], non_blocking=True)
        ev_in[j].record(copy)
        main.wait_event(ev_in[j])
        main.wait_event(ev_out[j])  # the previous read-back of this layer's output is done
        graphs[j].replay()
        ev_done[j].record(main)
        back.wait_event(ev_done[j])
        with torch.cuda.stream(back):
            ho_b[j].copy_(lay.out, non_blocking=True)
        ev_out[j].record(back)

    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize(dev)

    def e2e_timed(i):
        if i == 0:
            copy.wait_stream(main)  # the first copy follows the start event
        e2e_step(i)
        if i == args.steps - 1:
            main.wait_stream(back)  # the end event follows the last read-back

    ms_e2e = timed(torch, dev, e2e_timed, args.steps, dist, preroll=False)
    h2d = hio_b[0].numel() * 2
    d2h = ho_b[0].numel() * 2
    return NS(ms_step=ms / args.steps, ms_layer_graphs=ms_layer_graphs / args.steps,
              ms_host_paced=ms_host_paced / args.steps, ms_e2e=ms_e2e / args.steps, ms_attn=ms_attn,
              alg_bytes=alg_bytes, staged=staged * hk, hist_token_heads=hist * hk, h2d=h2d, d2h=d2h,
              launches=launches_per_step * args.steps, clocks=clk, layers=layers, impl=impl, graphs=graphs,
              timed_graph=timed_graph, warm_graph=warm_graph)


def shifted_table(torch, bt, pages):
    """Block-table rows starting `pages` pages in (zero padded): a history
    shard's own view of the request's pages."""
    out = torch.zeros_like(bt)
    out[:, :bt.shape[1] - pages] = bt[:, pages:]
    return out


def run_split_kv(torch, dev, args, dist, plan, group):
    """cfg3 with each request's history split across the two ranks of a KV-head
    group (8 ranks): the owner attends [0, 12288) with the current chunk, its
    partner [12288, 24576); the pair all-gathers the partial (O, LSE) over NCCL
    and both fold them with merge_slab.  Timed over 4 layers (> L2), checked
    against the rank's own single pass over the whole history."""
    from oscar_b200 import kernels, synthetic
    from oscar_b200.shards import page_shards

    lo, hi = page_shards(24576, 128, plan.splits)[plan.split]
    layers = []
    for li in range(4):
        full = synthetic.make_case([24576] * 8, [4] * 8, hk=GROUPS, group=GROUP_HQ, seed=1000 + li, device=dev)
        synthetic.fill_caches(full)
        del full.old_k, full.old_v
        c = slice_case(torch, full, plan.g0, plan.g1, 0, 8)
        del full
        n = c.q.shape[0]
        obuf = torch.empty(plan.splits, n, GROUP_HQ, D, dtype=torch.float32, device=dev)
        lbuf = torch.empty(plan.splits, n, GROUP_HQ, dtype=torch.float32, device=dev)
        layers.append(NS(c=c, bt_tail=shifted_table(torch, c.bt, lo // 128), obuf=obuf, lbuf=lbuf))

    def partial(lay):
        c = lay.c
        if plan.split == 0:
            return kernels.slab_attention(c.q, c.k_new, c.v_new, c.kc, c.vc, c.bt, c.qsl, [hi + 4] * 8, c.scale,
                                          c.stage)
        return kernels.slab_attention_shard(c.q, c.kc, c.vc, lay.bt_tail, c.qsl, [hi - lo] * 8, c.scale, c.stage)

    def exchange(lay, o, lse):
        dist.all_gather_into_tensor(lay.obuf, o, group=group)
        dist.all_gather_into_tensor(lay.lbuf, lse, group=group)
        out, l_out = lay.obuf[0], lay.lbuf[0]
        for p in range(1, plan.splits):
            kernels.merge_slab(out, l_out, lay.obuf[p], lay.lbuf[p], 0, None)
        return out, l_out

    def step(i):
        lay = layers[i % 4]
        exchange(lay, *partial(lay))

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize(dev)
    ms = timed(torch, dev, step, args.steps, dist) / args.steps
    parts = [partial(lay) for lay in layers]
    torch.cuda.synchronize(dev)
    ms_attn = timed(torch, dev, lambda i: partial(layers[i % 4]), args.steps, dist) / args.steps
    ms_xchg = timed(torch, dev, lambda i: exchange(layers[i % 4], *parts[i % 4]), args.steps, dist) / args.steps
    # check: the merged result equals this rank's single pass over the whole history
    err_o = err_l = 0.0
    for lay, p in zip(layers, parts):
        out, l_out = exchange(lay, *p)
        c = lay.c
        ref_o, ref_l = kernels.slab_attention(c.q, c.k_new, c.v_new, c.kc, c.vc, c.bt, c.qsl, c.seqs, c.scale, c.stage)
        err_o = max(err_o, float(((out - ref_o).abs() - 2e-2 * ref_o.abs()).max()))
        err_l = max(err_l, float(((l_out - ref_l).abs() - 1e-3 * ref_l.abs()).max()))
    ok = err_o <= 2e-2 and err_l <= 1e-3
    assert kernels.device_error(dev) == 0
    return {"workload": "cfg3_mtp_8x24k, history split in two page-aligned shards per KV-head group",
            "ms_per_step": ms, "query_tokens_per_s": 32.0 / (ms * 1e-3), "ms_attention": ms_attn,
            "ms_exchange_and_merge": ms_xchg, "exchange_share": ms_xchg / ms,
            "exchange": "NCCL all_gather_into_tensor of (O fp32 [32, 6, 256], LSE [32, 6]) within the pair, "
                        "then merge_slab",
            "rank0_shard": [lo, hi], "check_vs_single_pass": {"ok": ok, "excess_abs_out": err_o,
                                                              "excess_abs_lse": err_l}}


def run_cfg4(torch, dev, args, dist, plan):
    """cfg4: 15360 new tokens (causal) on 9256 tokens of INT2 history, Hq 24 /
    Hk 4.  KV-head groups over up to 4 ranks; on 8, each rank of a pair takes
    3 of its group's 6 query heads with the KV head replicated (vLLM's layout
    at tensor-parallel 8 over 4 KV heads).  Attention pass (tensor-core
    continuation kernel, pre-pass on) and the whole layer step through the
    backend; compute-bound (the 189 MB of queries exceed L2)."""
    from oscar_b200 import kernels, synthetic

    full = synthetic.make_case([9256], [15360], hk=GROUPS, group=GROUP_HQ, seed=31, device=dev)
    synthetic.fill_caches(full)
    del full.old_k, full.old_v
    c = slice_case(torch, full, plan.g0, plan.g1, 0, 1)
    del full
    hk = plan.g1 - plan.g0
    heads = slice(0, GROUP_HQ * hk)
    if plan.splits > 1:
        per = GROUP_HQ // plan.splits
        heads = slice(plan.split * per, (plan.split + 1) * per)
    q = c.q[:, heads].contiguous()
    hq = q.shape[1]
    args_attn = (q, c.k_new, c.v_new, c.kc, c.vc, c.bt, c.qsl, c.seqs, c.scale, c.stage)
    # --workspace-mib bounds this pass too: 0 times the per-CTA dequantisation path (no pre-pass)
    ws = kernels.DEFAULT_WORKSPACE_BYTES if args.workspace_mib is None else args.workspace_mib * 1024 * 1024
    attn = lambda i: kernels.slab_attention(*args_attn, workspace_bytes=ws)  # noqa: E731
    for _ in range(2):
        attn(0)
    torch.cuda.synchronize(dev)
    steps = max(3, min(args.steps, 10))
    ms_attn = timed(torch, dev, attn, steps, dist) / steps
    flops_rank = synthetic.attention_flops([9256], [15360], hq, D)
    flops = synthetic.attention_flops([9256], [15360], GROUPS * GROUP_HQ, D)
    check = None
    if plan.splits > 1:
        o3, l3 = attn(0)
        o6, l6 = kernels.slab_attention(c.q, c.k_new, c.v_new, c.kc, c.vc, c.bt, c.qsl, c.seqs, c.scale, c.stage,
                                        workspace_bytes=ws)
        check = {"vs_rank_full_group": bool(torch.allclose(o3, o6[:, heads], atol=2e-2, rtol=2e-2)
                                            and torch.allclose(l3, l6[:, heads], atol=1e-3, rtol=1e-3))}
    # the layer step through the backend (rotations, INT2 store of the chunk, staging, attention, output rotation)
    impl = make_backend(hk, args, hq)
    rk, rv = qr_pair(torch, 31, dev)
    layer = NS(layer_name="model.layers.3.self_attn.attn", _oscar_rots=(rk, rv))
    cache = (c.kc, c.vc)
    impl._set_caches(cache)
    impl._ensure_staging(layer, cache)
    pos = torch.arange(9256, 9256 + 15360, device=dev)
    slots = c.bt[0, pos // 128].long() * 128 + pos % 128
    md = NS(num_actual_tokens=15360, slot_mapping=slots, query_start_loc_cpu=torch.tensor(c.qsl),
            seq_lens_list=c.seqs, block_tables=c.bt, query_start_loc=torch.tensor(c.qsl, dtype=torch.int32, device=dev),
            seq_lens=torch.tensor(c.seqs, dtype=torch.int32, device=dev))
    out = torch.empty(15360, hq * D, dtype=torch.bfloat16, device=dev)
    fwd = lambda i: impl.forward(layer, q, c.k_new, c.v_new, cache, md, output=out)  # noqa: E731
    fwd(0)
    torch.cuda.synchronize(dev)
    ms_layer = timed(torch, dev, fwd, steps, dist) / steps
    assert kernels.device_error(dev) == 0
    _, peak_burst, peak_sus, src = load_peaks()
    tf = flops / (ms_attn * 1e-3) / 1e12
    return {"workload": "cfg4_continuation: 15360 new + 9256 INT2 history, Hq 24 / Hk 4",
            "workspace_bytes": ws, "ms_attention": ms_attn, "tflops": tf, "frac_bf16_burst": tf / peak_burst / dist_world(dist),
            "frac_bf16_sustained": tf / peak_sus / dist_world(dist), "peak_source": src,
            "rank_tflops": flops_rank / (ms_attn * 1e-3) / 1e12, "ms_layer_step": ms_layer,
            "layer_step": "backend.forward, eager: q/k/v rotations, clip + INT2 store of 15360 tokens, staging "
                          "write, attention, output rotation",
            "partition": f"rank 0: KV-head groups [{plan.g0}, {plan.g1}), query heads {heads.start}..{heads.stop - 1}",
            "check": check}


def dist_world(dist):
    return 1 if dist is None else dist.get_world_size()


def sum_over_ranks(torch, dist, dev, value):
    if dist is None:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t)
    return float(t.item())


def cfg5_schedule(n_steps=4, seed=5):
    """The cfg5 request set and a cycle of MTP steps with reject rewrites:
    step s writes lengths[s][r] tokens after base[s][r] accepted ones, then
    1..lengths tokens are accepted and the next step rewrites the rest
    (tests/test_streaming_backend.py:89-145 in the reference).  After the last
    step the cycle starts again from the first (a rollback: the same slots are
    rewritten with new values)."""
    from oscar_b200 import synthetic

    spec = synthetic.BASELINE_CONFIGS["cfg5_mixed_64"]
    prefixes = list(spec["prefixes"])
    rng = np.random.default_rng(seed)
    base = list(prefixes)
    steps = []
    for s in range(n_steps):
        lengths = list(spec["lengths"]) if s == 0 else [int(x) for x in rng.integers(1, 5, len(base))]
        steps.append((list(base), lengths))
        base = [b + int(rng.integers(1, ln + 1)) for b, ln in zip(base, lengths)]
    return prefixes, steps


def cfg5_requests(prefixes, plan):
    """Requests [r0, r1) of this rank: all of them, or (8 ranks) one of the
    halves of equal history."""
    if plan.splits == 1:
        return 0, len(prefixes)
    cum = np.cumsum(prefixes)
    bounds = [0] + [int(np.searchsorted(cum, cum[-1] * (i + 1) / plan.splits)) + 1
                    for i in range(plan.splits - 1)] + [len(prefixes)]
    return bounds[plan.split], bounds[plan.split + 1]


def run_cfg5(torch, dev, args, dist, plan, n_layers=16):
    """cfg5: 64 mixed requests (lognormal histories), 1-4-token MTP steps with
    reject rewrites, 16 stacked FULL layers with their own rotations, Hq 24 /
    Hk 4, through backend.forward.  Device time replays one CUDA graph per
    step geometry (16 layer forwards each); the eager figure is the host-paced
    backend API with the geometry changing every step."""
    from oscar_b200 import kernels, synthetic
    from oscar_b200.graphs import GraphedSequence

    prefixes, sched = cfg5_schedule()
    r0, r1 = cfg5_requests(prefixes, plan)
    hk = plan.g1 - plan.g0
    hq = GROUP_HQ * hk
    impl = make_backend(hk, args)
    gen = torch.Generator(device=dev).manual_seed(77)
    geoms = []
    for base, lengths in sched:
        base, lengths = base[r0:r1], lengths[r0:r1]
        qsl = [0]
        for ln in lengths:
            qsl.append(qsl[-1] + ln)
        n = qsl[-1]
        io = torch.randn(n * (hq + 2 * hk) * D, generator=gen, device=dev).bfloat16()
        q = io[:n * hq * D].view(n, hq, D)
        k = io[n * hq * D:n * (hq + hk) * D].view(n, hk, D)
        v = io[n * (hq + hk) * D:].view(n, hk, D)
        out = torch.empty(n, hq * D, dtype=torch.bfloat16, device=dev)
        geoms.append(NS(base=base, lengths=lengths, qsl=qsl, seqs=[b + ln for b, ln in zip(base, lengths)], q=q, k=k,
                        v=v, out=out))
    layers = []
    for li in range(n_layers):
        full = synthetic.make_case(prefixes, sched[0][1], hk=GROUPS, group=GROUP_HQ, seed=2000 + li, device=dev,
                                   compact=True, headroom=16)
        synthetic.fill_caches(full)
        del full.old_k, full.old_v
        c = slice_case(torch, full, plan.g0, plan.g1, r0, r1)
        del full
        rk, rv = qr_pair(torch, 100 + li, dev)
        layer = NS(layer_name=f"model.layers.{li}.self_attn.attn", _oscar_rots=(rk, rv))
        cache = (c.kc, c.vc)
        impl._set_caches(cache)
        impl._ensure_staging(layer, cache)
        for dst, src in zip((layer._oscar_stage_k, layer._oscar_stage_v, layer._oscar_slot_owner), c.stage):
            dst.copy_(src)
        mds = []
        for g in geoms:
            pos_r = [torch.arange(b, b + ln, device=dev) for b, ln in zip(g.base, g.lengths)]
            slots = torch.cat([c.bt[r, p // 128].long() * 128 + p % 128 for r, p in enumerate(pos_r)])
            mds.append(NS(num_actual_tokens=len(slots), slot_mapping=slots, query_start_loc_cpu=torch.tensor(g.qsl),
                          seq_lens_list=g.seqs, block_tables=c.bt,
                          query_start_loc=torch.tensor(g.qsl, dtype=torch.int32, device=dev),
                          seq_lens=torch.tensor(g.seqs, dtype=torch.int32, device=dev)))
        layers.append(NS(layer=layer, cache=cache, mds=mds, bt=c.bt))
    torch.cuda.synchronize(dev)
    S = len(geoms)
    pool = torch.cuda.graph_pool_handle()
    graphs = [GraphedSequence([(impl, lay.layer, g.q, g.k, g.v, lay.cache, lay.mds[s], g.out) for lay in layers],
                              pool=pool) for s, g in enumerate(geoms)]

    def eager(i):
        g = geoms[i % S]
        for lay in layers:
            impl.forward(lay.layer, g.q, g.k, g.v, lay.cache, lay.mds[i % S], output=g.out)

    for i in range(max(args.warmup, 3)):
        graphs[i % S].replay()
    torch.cuda.synchronize(dev)
    assert kernels.device_error(dev) == 0
    steps = max(args.steps, 2 * S)
    ms = timed(torch, dev, lambda i: graphs[i % S].replay(), steps, dist) / steps
    eager(0)
    ms_eager = timed(torch, dev, eager, steps, dist, preroll=False) / steps
    assert kernels.device_error(dev) == 0
    # algorithmic bytes of a step: packed history of every (request, KV head, layer) + staged fp32 rows
    hist_th = sum(sum(g.base) for g in geoms) / S * hk * n_layers
    staged = 0
    for lay in layers:
        owner = lay.layer._oscar_slot_owner.reshape(-1)
        rows = owner.numel() // 128
        g = geoms[0]
        for r, b in enumerate(g.base):
            pos = torch.arange(b, device=dev)
            blk = lay.bt[r, pos // 128].long()
            staged += int((owner[(blk % rows) * 128 + pos % 128] == blk).sum())
    alg = BYTES_PER_TOKEN_HEAD * hist_th + BYTES_PER_STAGED * staged * hk
    alg_all = sum_over_ranks(torch, dist, dev, alg)
    tokens = sum(sum(ln) for _, ln in sched) / S
    hbm, _, _, src = load_peaks()
    gbs = alg_all / (ms * 1e-3) / 1e9
    return {"workload": f"cfg5_mixed_64: 64 requests (lognormal history, median 4096, 1024..32768), 1-4 MTP tokens, "
                        f"{S}-step reject-rewrite cycle, {n_layers} layers, Hq 24 / Hk 4",
            "ms_per_step": ms, "query_tokens_per_s": tokens / (ms * 1e-3), "ms_per_layer": ms / n_layers,
            "gbs": gbs, "hbm_frac": gbs / (hbm * dist_world(dist)), "peak_source": src,
            "algorithmic_bytes_per_step": alg_all, "ms_per_step_eager_host_paced": ms_eager,
            "step_mode": "one CUDA graph per step geometry (16 backend forwards), replayed in turn",
            "partition": f"rank 0: KV-head groups [{plan.g0}, {plan.g1}), requests [{r0}, {r1})"}


def attention_traffic(hist_token_heads):
    """DRAM bytes of one attention pass from the committed ncu capture:
    measured bytes per history token-head (ncu's dram__bytes_read.sum +
    dram__bytes_write.sum over the decode kernel and its combine) times this
    launch's token-heads; None without a capture."""
    f = ROOT / "profiles" / "attention_traffic.json"
    if not f.exists():
        return None
    per = json.loads(f.read_text()).get("bytes_per_token_head")
    return None if per is None else per * hist_token_heads


def run_gpu(args):
    import torch

    from oscar_b200 import kernels

    world, rank, dist, dev = init_dist()
    plan = shard_plan(world, rank, 8)
    pair = pair_groups(dist, world)
    if args.only:
        # one secondary workload alone (profiling runs): its JSON object, no headline
        fn = {"cfg4": lambda: run_cfg4(torch, dev, args, dist, plan),
              "cfg5": lambda: run_cfg5(torch, dev, args, dist, plan),
              "split_kv": lambda: run_split_kv(torch, dev, args, dist, plan, pair)}[args.only]
        if args.only == "split_kv" and pair is None:
            raise SystemExit("--only split_kv needs 8 ranks (pairs of ranks per KV-head group)")
        line = fn()
        assert kernels.device_error(dev) == 0
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"only": args.only, **line}), flush=True)
        return
    head = run_headline(torch, dev, args, world, rank, dist, plan)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline_sample(head.layers[0], plan)
        except Exception as exc:  # keep the bench line if the sample fails
            cpu = {"value": None, "unit": UNIT, "cores": 1, "kind": "port", "sample": f"failed: {exc}"}
    del head.layers, head.impl, head.graphs, head.timed_graph, head.warm_graph
    torch.cuda.empty_cache()
    secondary = {}
    if not args.no_secondary:
        if pair is not None:
            secondary["cfg3_split_kv"] = run_split_kv(torch, dev, args, dist, plan, pair)
            torch.cuda.empty_cache()
        secondary["cfg4_continuation"] = run_cfg4(torch, dev, args, dist, plan)
        torch.cuda.empty_cache()
        secondary["cfg5_mixed_16l"] = run_cfg5(torch, dev, args, dist, plan)
    assert kernels.device_error(dev) == 0

    hbm, _, _, src = load_peaks()
    achieved = head.alg_bytes / (head.ms_attn * 1e-3) / 1e9
    tokens = 32  # the global step: 8 requests x 4 MTP tokens (all KV-head groups)
    result = {
        "metric": METRIC, "value": tokens / (head.ms_step * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head.ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded; no public dataset)",
        "config": workload_config(args.layers, plan, world),
        "step_latency_us": head.ms_step * 1e3,
        "step_mode": "one CUDA graph of the timed steps' layer forwards (oscar_b200.graphs.GraphedSequence), "
                     "replayed once; max over ranks",
        "ms_per_step_graph_per_layer": head.ms_layer_graphs,
        "ms_per_step_eager_host_paced": head.ms_host_paced,
        "e2e": {"value": tokens / (head.ms_e2e * 1e-3), "unit": UNIT, "h2d_bytes_per_step": head.h2d * world,
                "d2h_bytes_per_step": head.d2h * world, "ms_per_step": head.ms_e2e,
                "path": "per-layer GraphedForward replay of backend.forward; every step copies q/k/v in from one "
                        "pinned host buffer and the output back to pinned host memory, on copy streams that "
                        "overlap the neighbouring steps; one host wait at the end"},
        "gpu_launches": int(head.launches),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "traffic": attention_traffic(head.hist_token_heads),
                     "kernel": "slab attention pass (decode_tc_kernel + tc_combine_kernel), rank 0",
                     "launch_us": head.ms_attn * 1e3, "algorithmic_bytes": head.alg_bytes,
                     "staged_token_heads": head.staged, "history_token_heads": head.hist_token_heads,
                     "peak_source": src},
        "clocks": head.clocks,
    }
    if cpu is not None:
        result["cpu_baseline"] = cpu
    if secondary:
        result["secondary"] = secondary
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


# ---------------------------------------------------------------------------
# reference arm: the reference algorithm's CPU restatement on the host cores
_REF = {}


def _ref_init():
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(1)
    except Exception:
        pass


def _ref_attend(unit):
    """Attention of one (request, KV-head group) unit of the step."""
    from oracle import oscar_oracle as orc

    d = _REF
    req, g = divmod(unit, GROUPS)
    a, b = d["qsl"][req], d["qsl"][req + 1]
    hs = slice(GROUP_HQ * g, GROUP_HQ * (g + 1))
    sk, sv, owner = d["stage"]
    out, _ = orc.streaming_attention(d["qr"][a:b, hs], d["kr"][a:b, g:g + 1], d["vr"][a:b, g:g + 1],
                                     d["k8"][:, :, g:g + 1], d["v8"][:, :, g:g + 1], d["bt"][req:req + 1], [0, b - a],
                                     [d["seqs"][req]], d["scale"], (sk[:, :, g:g + 1], sv[:, :, g:g + 1], owner))
    return unit, out


def run_reference(args):
    """The same layer step (cfg3, Hq 24 / Hk 4, all 32 (request, KV-head group)
    units) on the oracle: rotate, clip, INT2 store and staging write of the
    step's tokens in the parent, the 32 attention units spread over forked
    worker processes (one BLAS thread each), then the output rotation.  Under
    torchrun only rank 0 runs; the others exit without work."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import multiprocessing as mp

    import torch

    from oracle import oscar_oracle as orc
    from oscar_b200 import synthetic

    prefixes, lengths = [24576] * 8, [4] * 8
    case = synthetic.make_case(prefixes, lengths, hk=GROUPS, group=GROUP_HQ, seed=1000)
    k8 = case.kc.view(torch.uint8).numpy().copy()
    v8 = case.vc.view(torch.uint8).numpy().copy()
    orc.store(case.old_k.numpy(), case.old_v.numpy(), k8, v8, case.slots.numpy())
    del case.old_k, case.old_v
    g = torch.Generator().manual_seed(7)
    rk = torch.linalg.qr(torch.randn(D, D, generator=g)).Q.numpy().astype(np.float32)
    rv = torch.linalg.qr(torch.randn(D, D, generator=g)).Q.numpy().astype(np.float32)
    st = orc.Staging(128, GROUPS, D, 128, 256, 8192)
    sk, sv, owner = (t.numpy() for t in case.stage)
    st.stage_k[:], st.stage_v[:], st.owner[:] = sk, sv, owner
    q = case.q.float().numpy()
    kn = case.k_new.float().numpy()
    vn = case.v_new.float().numpy()
    slots = np.concatenate([case.bt[r].numpy()[np.arange(p, p + n) // 128].astype(np.int64) * 128
                            + np.arange(p, p + n) % 128 for r, (p, n) in enumerate(zip(prefixes, lengths))])
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    units = 8 * GROUPS
    nproc = max(1, min(cores, units))

    def host_write():
        kr_u, vr_u = kn @ rk, vn @ rv
        orc.store(orc.clip_only(kr_u, 0.96), orc.clip_only(vr_u, 0.92), k8, v8, slots)
        st.write(kn, vn, rk, rv, slots, case.qsl, case.seqs, len(slots))
        return orc.round_bf16(q @ rk), orc.round_bf16(kr_u), orc.round_bf16(vr_u)

    # one write before forking: the workers inherit the written caches and
    # staging, and every later step writes the same bytes again (the MTP slots repeat)
    qr, kr, vr = host_write()
    _REF.update(k8=k8, v8=v8, bt=case.bt.numpy(), qsl=case.qsl, seqs=case.seqs, scale=case.scale, stage=st.tuple(),
                qr=qr, kr=kr, vr=vr)
    ctx = mp.get_context("fork")  # this arm never initialises CUDA

    def one_step(pool):
        host_write()
        out = np.empty((q.shape[0], GROUPS * GROUP_HQ, D), np.float32)
        for unit, o in pool.imap_unordered(_ref_attend, range(units)):
            req, grp = divmod(unit, GROUPS)
            out[case.qsl[req]:case.qsl[req + 1], GROUP_HQ * grp:GROUP_HQ * (grp + 1)] = o
        return orc.round_bf16(out @ rv.T)

    with ctx.Pool(nproc, initializer=_ref_init) as pool:
        for _ in range(args.warmup):
            one_step(pool)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            one_step(pool)
        dt = (time.perf_counter() - t0) / args.steps
    value = 32 / dt
    plan = shard_plan(1, 0, 8)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; no public dataset)",
        "config": workload_config(args.layers, plan, 1),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": nproc, "kind": "port",
                         "sample": f"the whole cfg3 layer step (8 x 24576 history + 4 MTP tokens, Hq 24 / Hk 4) on "
                                   f"the numpy oracle, its {units} (request, KV-head group) attention units over "
                                   f"{nproc} forked processes; 1 layer (the CPU reads its caches from DRAM either "
                                   f"way)"},
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

