"""Blended-prefill benchmark: CacheBlend selective recompute at Mistral-7B shape.

Workload (one step = one blended prefill of one request, per GPU): Mistral-7B
architecture with random-init bf16 weights (32 layers, hidden 4096, 32 q / 8 KV
heads, head_dim 128, rope_theta 1e6, vocab 32000); prompt = 6 chunks x 1024
uniform-random token ids + a 64-token query chunk (S = 6208); chunk K/V
precomputed per chunk (untimed, like the reference's collect phase);
recompute ratio 0.15 (k = 931), check layer 1.  Synthetic ids stand in for the
reference's musique passages (about 6-7K tokens per prompt).

  value   fused prompt tokens / s over all ranks, device-timed (CUDA events)
          over K steps of ``fuse_selective`` + argmax of the last position,
          inputs resident in HBM
  e2e     the same through the public API with the token ids copied from
          pinned host memory and the first decoded token read back each step
  roofline  the dominant libcbk kernel (partial attention): algorithmic FLOPs
          of its launches / their CUDA-event time inside the timed region

Multi-GPU: one process per GPU (torchrun), each rank runs its own requests
(independent units, no data-path collective); the step time is the max over
ranks.  ``--impl reference`` times the reference's algorithm on the host CPU
(the oracle restatement) for the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "cacheblend-hf-v7_b200"))
sys.path.insert(0, ROOT)

METRIC = "blended-prefill TTFT (ms) & tokens/s at Mistral-7B 7K ctx; KV-kernel HBM GB/s"
MISTRAL_7B = dict(vocab_size=32000, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                  num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=1e6,
                  rms_norm_eps=1e-5, max_position_embeddings=32768, sliding_window=None)
N_CHUNKS, CHUNK_LEN, QUERY_LEN, RATIO, CHECK_LAYER = 6, 1024, 64, 0.15, 1


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p["bf16_tflops_sustained"], "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


# ---------------------------------------------------------------------------
# clocks sampler
# ---------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=5)
        except Exception:
            self.p.kill()
            return None
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
def build_request(model, cb, seed, device):
    import torch
    gen = torch.Generator().manual_seed(seed)
    lens = [CHUNK_LEN] * N_CHUNKS + [QUERY_LEN]
    ids = [torch.randint(0, MISTRAL_7B["vocab_size"], (n,), generator=gen).tolist() for n in lens]
    chunks = [cb.Chunk(text=f"r{seed}c{i}", token_ids=t, chunk_id=cb.chunker._stable_id(f"r{seed}c{i}", t))
              for i, t in enumerate(ids)]
    return chunks


def build_model(device):
    import torch
    from transformers import MistralConfig, MistralForCausalLM
    cfg = MistralConfig(**MISTRAL_7B)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    with torch.device(device):
        model = MistralForCausalLM(cfg).to(torch.bfloat16)
    return model.eval()


def attn_flops(idx_list, S, Hq, D, ck, n_layers):
    """Algorithmic FLOPs of the partial-attention launches of one step:
    4 * Hq * D * sum(pos + 1) per layer (QK^T and PV over the causal prefix)."""
    sel = sum(int(p) + 1 for p in idx_list)
    dense = S * (S + 1) // 2
    return 4 * Hq * D * (dense * ck + sel * (n_layers - ck))


def _short_kernels_alone(lw, chunks, store, idx, S, cfg, device, hbm_peak, reps=31):
    """The step's short HKVD and RoPE/scatter calls timed on their own: the same
    shapes, selection (idx) and chunk K, reps calls back to back in one CUDA graph,
    CUDA events around its replays.  Inside the step each call sits between event
    nodes and shares the GPU with the assemble kernel on the side stream; these
    figures show the kernels' own rates at this size."""
    import torch
    from cacheblend import ops
    from cacheblend.fusor import _store_entries
    from cacheblend.rope import rope_table_for
    D, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    kv = Hkv * D
    k_sel = idx.numel()
    g = torch.Generator(device=device).manual_seed(5)
    qkv = torch.randn((k_sel, (Hq + 2 * Hkv) * D), generator=g, device=device).to(torch.bfloat16)
    q, kr, vr = qkv[:, :Hq * D], qkv[:, Hq * D:Hq * D + kv], qkv[:, Hq * D + kv:]
    fk = torch.zeros((S, kv), dtype=torch.bfloat16, device=device)
    fv = torch.zeros_like(fk)
    rope_sel = rope_table_for(lw, S, device).index_select(0, idx)
    q_out = torch.empty((k_sel, Hq * D), dtype=torch.bfloat16, device=device)
    table = ops.ChunkTable(_store_entries(store, chunks, "bench"), [CHECK_LAYER], device)
    kn = torch.randn((S, kv), generator=g, device=device).to(torch.bfloat16)
    ws = torch.empty((int(ops.N.LIB.cbk_hkvd_workspace_bytes(S)) // 4,), dtype=torch.float32, device=device)

    def per_call_us(fn):
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            fn()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                for _ in range(reps):
                    fn()
        torch.cuda.current_stream(device).wait_stream(side)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(5):
            graph.replay()
        b.record()
        torch.cuda.synchronize()
        del graph
        return a.elapsed_time(b) * 1e3 / (5 * reps)

    out = {}
    for name, fn, nbytes in (
            ("rope_scatter", lambda: ops.rope_scatter(q, kr, vr, idx, False, S, Hq, Hkv, D, rope_sel, fk, fv,
                                                      q_out=q_out, table_by_row=True),
             k_sel * (Hq + 2 * Hkv) * D * 2 * 2),
            ("hkvd_select", lambda: ops.hkvd_select(kn, table, CHECK_LAYER, k_sel, True, workspace=ws),
             2 * S * kv * 2 + S * 4)):
        us = per_call_us(fn)
        gbs = nbytes / (us * 1e-6) / 1e9
        out[name] = {"us_per_call": round(us, 2), "GB/s": round(gbs, 1), "frac_hbm": round(gbs / hbm_peak, 3),
                     "how": f"{reps} calls of one sparse layer's shapes back to back in a CUDA graph"}
    return out


def _torch_restatement_gpu(model, chunks, store, idx, S, device, steps=3):
    """Context for the kernels: the reference's blended prefill restated with stock
    torch ops (concat, masks, repeat_interleave'd K/V, SDPA, index_put; the module
    tests/ref_torch.py, which the end-to-end tests compare against) in bf16 on the
    same GPU, plus its HKVD the same way (fp32 difference, square, sum; topk; sort;
    the force-include check on the host).  The selection is the device's own, and
    only the selected rows' logits are formed (the reference's dense (1, S, V)
    logits are not), so this is a lower bound on the reference's own GPU time."""
    import torch
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import ref_torch
    from cacheblend.fusor import _store_entries
    entries = _store_entries(store, chunks, "bench")
    ids = torch.tensor([t for c in chunks for t in c.token_ids], device=device)
    kv = model.config.num_key_value_heads * (model.config.hidden_size // model.config.num_attention_heads)
    k_old = torch.cat([e["K"][CHECK_LAYER] for e in entries], dim=1)[0]
    k_new = (k_old.float() + 0.05 * torch.randn(k_old.shape, device=device,
                                                generator=torch.Generator(device=device).manual_seed(3))).to(k_old.dtype)
    k_sel = idx.numel()

    def one():
        dev = ((k_new.float() - k_old.float()) ** 2).sum(-1)
        sel = torch.sort(torch.topk(dev, k_sel).indices).values
        if int(sel[-1].item()) != S - 1:                       # force-include on the host
            sel = torch.sort(torch.cat([sel[1:], torch.tensor([S - 1], device=device)])).values
        return ref_torch.selective_logits(model, ids, entries, idx, CHECK_LAYER)

    one()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        one()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    return {"ms_per_step": round(ms, 3), "tokens_per_s": round(S / (ms * 1e-3), 1), "steps": steps,
            "how": "the reference's steps in stock torch ops on the same GPU (tests/ref_torch.py + torch HKVD), "
                   "bf16, the same selection, selected-row logits only; CUDA events around the steps"}


def run_ours(args):
    import torch
    import torch.distributed as dist
    import cacheblend as cb
    from cacheblend._timing import TIMES

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    model = build_model(device)
    lw = cb.LayerwiseModel.from_hf(model)
    reqs = [build_request(model, cb, seed=1000 * rank + r, device=device) for r in range(args.requests)]
    if args.kv_arena:
        kv_dim = MISTRAL_7B["num_key_value_heads"] * MISTRAL_7B["head_dim"]
        n_tok = sum(c.length for chunks in reqs for c in chunks)
        store = cb.KVArena(MISTRAL_7B["num_hidden_layers"], kv_dim, n_tok, device)
        for chunks in reqs:
            for c in chunks:
                cb.precompute_chunk_kv_into(lw, c, store)
    else:
        store = cb.KVStore()
        for chunks in reqs:
            for c in chunks:
                K, V = cb.precompute_chunk_kv(lw, c)
                store.put(c.chunk_id, K, V)
    S = sum(c.length for c in reqs[0])
    stream = torch.cuda.current_stream(device)

    dev_ids = [torch.tensor([t for c in chunks for t in c.token_ids], dtype=torch.int64, device=device)
               for chunks in reqs]

    use_graph = not args.no_cuda_graph

    def step(i, graph=use_graph):
        chunks = reqs[i % len(reqs)]
        logits = cb.fuse_selective(lw, chunks, store, recompute_ratio=RATIO, check_layer=CHECK_LAYER,
                                   input_ids=dev_ids[i % len(reqs)], cuda_graph=None if graph else False)
        return logits[0, -1].argmax()

    for i in range(args.warmup):          # (the first call of the geometry captures its CUDA graph)
        step(i)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def device_timed(fn):
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        t0.record(stream)
        for i in range(args.steps):
            fn(i)
        t1.record(stream)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(t0.elapsed_time(t1))

    # --- device-timed region: the public API call (a replayed CUDA graph) -----
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)
    torch.cuda.nvtx.range_push("timed")
    ms = device_timed(step)
    torch.cuda.nvtx.range_pop()
    clk = clocks.stop()

    # --- end to end through the public API (host ids in, first token out) -----
    pinned = [torch.tensor([t for c in chunks for t in c.token_ids], dtype=torch.int64).pin_memory()
              for chunks in reqs]
    e2e_ms = []
    barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        chunks = reqs[i % len(reqs)]
        a = time.perf_counter()
        logits = cb.fuse_selective(lw, chunks, store, recompute_ratio=RATIO, check_layer=CHECK_LAYER,
                                   input_ids=pinned[i % len(reqs)],          # H2D of this step's ids
                                   cuda_graph=None if use_graph else False)
        int(logits[0, -1].argmax().item())                                   # first token to host
        e2e_ms.append((time.perf_counter() - a) * 1e3)
    barrier()
    e2e_step = max_over_ranks(sum(e2e_ms) / len(e2e_ms))

    # --- the same steps launched kernel by kernel from Python (context) ----------
    for i in range(args.warmup):
        step(i, graph=False)
    torch.cuda.synchronize()
    eager_ms = device_timed(lambda i: step(i, graph=False))
    eager_res = {"ms_per_step": round(eager_ms / args.steps, 3),
                 "tokens_per_s": round(world * S * args.steps / (eager_ms * 1e-3), 1),
                 "how": "fuse_selective(cuda_graph=False): every kernel launched from Python"}

    # --- per-kernel device times inside the graph --------------------------------
    # A second capture of the same geometry with an external CUDA event around
    # every libcbk launch (event-record nodes of the graph); each replay is
    # followed by a synchronize and the events are read: each kernel's own
    # duration as the graph runs it, on its launch stream, with no host gaps.
    TIMES.reset()
    TIMES.active = True
    tg = cb.BlendGraph(lw, reqs[0], store, recompute_ratio=RATIO, check_layer=CHECK_LAYER, dense_logits=False)
    TIMES.active = False
    spans = list(TIMES.graph_spans)
    TIMES.reset()
    acc = {}
    inst_ms = 0.0
    for i in range(args.steps):
        a_ev = torch.cuda.Event(enable_timing=True)
        b_ev = torch.cuda.Event(enable_timing=True)
        a_ev.record(stream)
        tg.replay(reqs[i % len(reqs)], store, input_ids=dev_ids[i % len(reqs)])
        b_ev.record(stream)
        torch.cuda.synchronize()
        inst_ms += a_ev.elapsed_time(b_ev)
        TIMES.read_graph_spans(spans, acc)
    del tg
    kern = {name: (v[0], v[1]) for name, v in acc.items()}
    instrumented = {"ms_per_step": round(inst_ms / args.steps, 3), "event_spans_per_step": len(spans),
                    "note": "the graph with an event pair around every libcbk launch, replayed alone per step "
                            "(its step time against the plain graph's shows what the event nodes cost)"}
    # the graph's launches plus the dense-logits scatter fuse_selective runs after the replay
    launch_counts = {name: v[2] for name, v in acc.items()}
    launch_counts["scatter_rows"] = launch_counts.get("scatter_rows", 0) + args.steps

    # --- kernel accounting -----------------------------------------------------
    _, idx = cb.fuse_selective(lw, reqs[0], store, recompute_ratio=RATIO, check_layer=CHECK_LAYER,
                               return_hkvd_indices=True)
    idx_l = idx.cpu().tolist()
    cfg = model.config
    D, Hq, Hkv, L = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.num_hidden_layers
    kv_dim = Hkv * D
    hbm_peak, tf_burst, tf_sust, peak_src = load_peaks()
    # attention: sparse layers (selected rows) and dense layers before the check layer
    sel_sum = sum(int(p) + 1 for p in idx_l)
    n_sp, ms_sp = kern.get("partial_attn", (0, 0.0))
    n_de, ms_de = kern.get("partial_attn_dense", (0, 0.0))
    fl_sp = 4 * Hq * D * sel_sum                       # per sparse-layer call
    fl_de = 4 * Hq * D * (S * (S + 1) // 2)            # per dense-layer call
    n_attn = n_sp + n_de
    attn_ms = ms_sp + ms_de
    per_launch_flops = (n_sp * fl_sp + n_de * fl_de) / max(n_attn, 1)
    attn_avg_ms = attn_ms / max(n_attn, 1)
    achieved_tf = per_launch_flops / (attn_avg_ms * 1e-3) / 1e12 if n_attn else None
    tf_sp = fl_sp / (ms_sp / n_sp * 1e-3) / 1e12 if n_sp else None
    tf_de = fl_de / (ms_de / n_de * 1e-3) / 1e12 if n_de else None
    n_asm, asm_ms = kern.get("assemble_kv", (0, 0.0))
    asm_bytes = (L - CHECK_LAYER) * 2 * 2 * S * kv_dim * 2        # read chunk K/V + write fused K/V
    n_hk, hk_ms = kern.get("hkvd_select", (0, 0.0))
    hk_bytes = 2 * S * kv_dim * 2 + S * 4
    n_sc, sc_ms = kern.get("rope_scatter", (0, 0.0))
    k_sel = len(idx_l)
    sc_bytes_sparse = k_sel * (cfg.hidden_size + 2 * kv_dim) * 2 * 2      # read + write Q, K, V rows
    sc_bytes_dense = S * (cfg.hidden_size + 2 * kv_dim) * 2 * 2
    sc_bytes_step = CHECK_LAYER * sc_bytes_dense + (L - CHECK_LAYER) * sc_bytes_sparse

    def gbs(nbytes, calls, total_ms):
        if not calls:
            return None, None
        r = nbytes / (total_ms / calls * 1e-3) / 1e9
        return round(r, 1), round(r / hbm_peak, 3)
    traffic = None
    prof = os.path.join(ROOT, "profiles", "partial_attn_kernel_mistral7b_7k_blend_traffic.json")
    if os.path.exists(prof):
        try:
            traffic = json.load(open(prof)).get("bytes_per_launch")
        except Exception:
            traffic = None

    alone = _short_kernels_alone(lw, reqs[0], store, idx, S, cfg, device, hbm_peak)
    torch_ref = _torch_restatement_gpu(model, reqs[0], store, idx, S, device) if world == 1 else None

    launches = sum(launch_counts.values())
    res = {
        "metric": METRIC,
        "value": round(world * S * args.steps / (ms * 1e-3), 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3),
        "ttft_ms": round(ms / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (uniform-random token ids; random-init weights)",
        "config": {"workload": "mistral7b-7k-blend", "model": "Mistral-7B architecture, random init",
                   "chunks": f"{N_CHUNKS}x{CHUNK_LEN}+{QUERY_LEN}", "S": S, "recompute_ratio": RATIO,
                   "k_selected": k_sel, "check_layer": CHECK_LAYER, "global_batch": world,
                   "selection": {"min_pos": int(min(idx_l)), "median_pos": int(sorted(idx_l)[len(idx_l) // 2]),
                                 "frac_in_last_1088": round(sum(p >= S - 1088 for p in idx_l) / len(idx_l), 3)},
                   "requests_per_rank": args.requests, "parallelism": f"by-request x{world}",
                   "kv_store": "KVArena (one device pool)" if args.kv_arena else "KVStore (tensor per chunk and layer)",
                   "l2": "inputs larger than L2 (14.5 GB weights, 0.81 GB fused KV per step)"},
        "e2e": {"value": round(world * S / (e2e_step * 1e-3), 1), "unit": "tokens/s",
                "ttft_ms": round(e2e_step, 3), "h2d_bytes_per_step": S * 8, "d2h_bytes_per_step": 8},
        "roofline": {"kernel": "partial_attn_kernel", "bound": "tensor",
                     "achieved": round(achieved_tf, 1) if achieved_tf else None,
                     "peak": tf_sust, "unit": "TFLOP/s",
                     "frac": round(achieved_tf / tf_sust, 4) if achieved_tf else None,
                     "peak_kind": f"{peak_src} bf16 sustained (kernel timed inside a long step)",
                     "flops_per_launch": per_launch_flops, "calls": n_attn,
                     "avg_launch_ms": round(attn_avg_ms, 5), "traffic": traffic,
                     "traffic_src": ("dram bytes per launch read from the committed ncu summary "
                                     "profiles/partial_attn_kernel_mistral7b_7k_blend_traffic.json, not measured "
                                     "in this run") if traffic else None,
                     "timed_in": ("CUDA events captured as graph nodes around each launch, read after each of "
                                  f"{args.steps} replays of the step's graph")},
        "kernels": {
            "assemble_kv": {"calls": n_asm, "avg_ms": round(asm_ms / max(n_asm, 1), 4),
                            "bytes": asm_bytes,
                            "GB/s": round(asm_bytes / (asm_ms / max(n_asm, 1) * 1e-3) / 1e9, 1) if n_asm else None,
                            "frac_hbm": round(asm_bytes / (asm_ms / max(n_asm, 1) * 1e-3) / 1e9 / hbm_peak, 3) if n_asm else None},
            "hkvd_select": {"calls": n_hk, "avg_ms": round(hk_ms / max(n_hk, 1), 4), "bytes": hk_bytes,
                            "GB/s": gbs(hk_bytes, n_hk, hk_ms)[0], "frac_hbm": gbs(hk_bytes, n_hk, hk_ms)[1],
                            "alone": alone["hkvd_select"]},
            "rope_scatter": {"calls": n_sc, "avg_ms": round(sc_ms / max(n_sc, 1), 4),
                             "bytes_sparse_layer": sc_bytes_sparse, "bytes_per_step": sc_bytes_step,
                             "GB/s": gbs(sc_bytes_step / L, n_sc, sc_ms)[0],
                             "frac_hbm": gbs(sc_bytes_step / L, n_sc, sc_ms)[1],
                             "alone": alone["rope_scatter"]},
            "partial_attn_sparse": {"calls": n_sp, "avg_ms": round(ms_sp / max(n_sp, 1), 4),
                                    "flops_per_call": fl_sp,
                                    "TFLOP/s": round(tf_sp, 1) if tf_sp else None},
            "partial_attn_dense": {"calls": n_de, "avg_ms": round(ms_de / max(n_de, 1), 4),
                                   "flops_per_call": fl_de,
                                   "TFLOP/s": round(tf_de, 1) if tf_de else None},
            "hbm_peak_gbs": hbm_peak, "hbm_peak_kind": peak_src,
        },
        "gpu_launches": launches,
        "gpu_launches_note": ("libcbk launches of the timed steps: the launches captured in the step's graph "
                              "times the steps, plus the dense-logits scatter run after each replay"),
        "clocks": clk,
        "eager_launches": eager_res,
        "instrumented_graph": instrumented,
        "timed_path": ("fuse_selective default: a CUDA graph of the request geometry, captured on the first "
                       "call, replayed per step" if use_graph else "fuse_selective(cuda_graph=False)"),
    }
    if torch_ref is not None:
        res["gpu_torch_restatement"] = torch_ref
    if world == 1 and not args.no_cpu_baseline:       # host-core baseline: rank 0 at N=1 only
        res["cpu_baseline"] = cpu_baseline()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


# ---------------------------------------------------------------------------
# CPU baseline / reference arm: the oracle restatement of fuse_selective
# ---------------------------------------------------------------------------
class OracleBlend:
    """One blended prefill of the reference's algorithm on the host cores (the
    oracle restatement, numpy fp32, every core), as a list of units run in
    order: concat + the full layers before the check layer; the check layer
    (HKVD, top-K, force-include); one unit per sparse layer; the final norm +
    lm_head + dense logits.  Running every unit once is one whole prefill, and
    each unit's time is measured as it runs (nothing is extrapolated)."""

    def __init__(self, W, ids, ck_k, ck_v, n_layers):
        from oracle import model as om
        self.om, self.W, self.ids, self.ck_k, self.ck_v, self.L = om, W, ids, ck_k, ck_v, n_layers
        self.prep = self.state = self.result = None

    def units(self):
        om, W = self.om, self.W

        def prep():
            self.prep = om.selective_prepare(self.ids, self.ck_k, self.ck_v, W, CHECK_LAYER, self.L)

        def check():
            self.state = om.selective_check(self.prep, W, RATIO)
            self.prep = None

        def end():
            self.result = om.selective_end(self.state, W)
            self.state = None

        sparse = [lambda l=l: om.selective_layer(self.state, l, W, keep_cache=False)
                  for l in range(CHECK_LAYER + 1, self.L)]
        return [prep, check] + sparse + [end]


def _mem_available_gb():
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) / 2 ** 20
    except OSError:
        pass
    return 0.0


def _synthetic_oracle_inputs(seed=0):
    """Random-init Mistral-7B-shape weights (N(0, 0.02), unit norm weights) as
    oracle fp32 arrays, the 7-chunk request's ids and per-layer chunk K / V
    ~ N(0, 1).  With enough host memory every layer has its own weights (29
    GB); otherwise the sparse layers 2..31 share one weight set and one chunk
    K / V set (same shapes, so the same work per layer; a layer's weights are
    0.87 GB, far larger than the host caches, so sharing them does not make a
    layer faster).  Returns (W, ids, ck_k, ck_v, distinct)."""
    import numpy as np
    from oracle import model as om, threads
    c = MISTRAL_7B
    L = c["num_hidden_layers"]
    H, I, kvd = c["hidden_size"], c["intermediate_size"], c["num_key_value_heads"] * c["head_dim"]
    distinct = _mem_available_gb() >= 96
    n_sets = L if distinct else CHECK_LAYER + 2
    cfg = om.Config(c["vocab_size"], H, I, L, c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"],
                    c["rope_theta"], c["rms_norm_eps"])

    def w(seed_, *shape):
        r = np.random.default_rng(seed_)
        return r.standard_normal(shape, dtype=np.float32) * np.float32(0.02)

    def layer(l):
        b = 1000 * (l + 1) + seed
        return {"q": w(b, H, H), "k": w(b + 1, kvd, H), "v": w(b + 2, kvd, H), "o": w(b + 3, H, H),
                "gate": w(b + 4, I, H), "up": w(b + 5, I, H), "down": w(b + 6, H, I),
                "ln1": np.ones(H, np.float32), "ln2": np.ones(H, np.float32)}

    sets = threads.run([lambda l=l: layer(l) for l in range(n_sets)])
    W = om.Weights.__new__(om.Weights)
    W.cfg = cfg
    W.embed, W.lm_head = threads.run([lambda: w(seed + 1, c["vocab_size"], H), lambda: w(seed + 2, c["vocab_size"], H)])
    W.norm = np.ones(H, np.float32)
    W.layers = [sets[min(l, n_sets - 1)] for l in range(L)]
    W.inv_freq = __import__("oracle").hotpath.inv_freq(c["rope_theta"], c["head_dim"])
    rng = np.random.default_rng(seed + 3)
    lens = [CHUNK_LEN] * N_CHUNKS + [QUERY_LEN]
    ids = [rng.integers(0, c["vocab_size"], n) for n in lens]
    kv_sets = [[(rng.standard_normal((n, kvd), dtype=np.float32), rng.standard_normal((n, kvd), dtype=np.float32))
                for n in lens] for _ in range(n_sets)]
    ck_k = [[kv_sets[min(l, n_sets - 1)][i][0] for l in range(L)] for i in range(len(lens))]
    ck_v = [[kv_sets[min(l, n_sets - 1)][i][1] for l in range(L)] for i in range(len(lens))]
    return W, ids, ck_k, ck_v, distinct


def _oracle_sample_text(distinct, cores):
    return (f"the reference's fuse_selective restated by the oracle (numpy fp32, {cores} host threads) on the "
            f"Mistral-7B 7K workload (S = 6208, ratio 0.15, 32 layers, random-init weights"
            f"{'' if distinct else '; sparse layers 2..31 share one weight set'}); every unit of each "
            f"prefill (concat + layer 0, check layer + HKVD, 30 sparse layers, lm_head) timed, none extrapolated")


def cpu_baseline():
    """Host-core baseline for the N=1 line: one whole blended prefill of the
    reference's algorithm (oracle, every core), measured unit by unit."""
    W, ids, ck_k, ck_v, distinct = _synthetic_oracle_inputs()
    ob = OracleBlend(W, ids, ck_k, ck_v, MISTRAL_7B["num_hidden_layers"])
    t = time.perf_counter()
    for u in ob.units():
        u()
    ttft = time.perf_counter() - t
    S = sum(len(x) for x in ids)
    cores = _blas_threads()
    return {"value": round(S / ttft, 2), "unit": "tokens/s", "ttft_s": round(ttft, 3), "cores": cores,
            "kind": "port", "sample": "one prefill: " + _oracle_sample_text(distinct, cores)}


def _blas_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else 1
    except Exception:
        return os.cpu_count() or 1


def run_reference(args):
    """Reference arm: the reference's algorithm (oracle restatement, numpy on the
    host cores) on the same workload."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    # torchrun sets OMP_NUM_THREADS=1 for every rank; the reference arm runs on
    # rank 0 alone and may use every host core
    try:
        from threadpoolctl import threadpool_limits
        from oracle import threads
        limiter = threadpool_limits(limits=threads.n_threads())
    except Exception:
        limiter = None
    try:
        _run_reference(args)
    finally:
        if limiter is not None:
            limiter.restore_original_limits()


def _run_reference(args):
    """The K timed steps cover R = ceil(K / U) whole blended prefills of U units
    each, split into K consecutive runs of units (step i runs units
    [i*R*U/K, (i+1)*R*U/K) of the sequence), so every layer of every reported
    prefill is timed; value = R * S / (time of the K steps).  The W warm-up
    steps run one sparse-layer unit each on a separate prefill."""
    W, ids, ck_k, ck_v, distinct = _synthetic_oracle_inputs()
    L = MISTRAL_7B["num_hidden_layers"]
    S = sum(len(x) for x in ids)
    warm = OracleBlend(W, ids, ck_k, ck_v, L)
    wu = warm.units()
    wu[0]()
    wu[1]()
    for i in range(args.warmup):
        wu[2 + i % (L - CHECK_LAYER - 1)]()
    del warm, wu
    U = L + 2
    R = -(-args.steps // U)
    seq = []
    for _ in range(R):
        seq += OracleBlend(W, ids, ck_k, ck_v, L).units()
    bounds = [i * R * U // args.steps for i in range(args.steps + 1)]
    step_s = []
    t_all = time.perf_counter()
    for i in range(args.steps):
        t = time.perf_counter()
        for u in seq[bounds[i]:bounds[i + 1]]:
            u()
        step_s.append(time.perf_counter() - t)
    total = time.perf_counter() - t_all
    value = round(R * S / total, 2)
    cores = _blas_threads()
    sample = (f"{R} whole prefill(s) over the {args.steps} timed steps (each step runs the next "
              f"{R * U / args.steps:.2f} of the {U} units in order): " + _oracle_sample_text(distinct, cores))
    print(json.dumps({
        "metric": METRIC, "impl": "reference", "value": value, "unit": "tokens/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total * 1e3 / args.steps, 1), "ttft_ms": round(total * 1e3 / R, 1),
        "step_ms": [round(x * 1e3, 1) for x in step_s], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "mistral7b-7k-blend", "S": S, "recompute_ratio": RATIO,
                   "check_layer": CHECK_LAYER, "parallelism": "host CPU", "host_mem_available_gb":
                   round(_mem_available_gb(), 1)},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------
# kernel-level workloads (no model): KV kernels at the microbench shape, and the
# partial-attention kernel at the Mistral-7B sparse-layer shape
# ---------------------------------------------------------------------------
def _timed(fn, steps, warmup, device):
    import torch
    from cacheblend._timing import TIMES
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    clocks = Clocks(device.index or 0)
    clocks.start()
    time.sleep(0.3)
    TIMES.reset()
    TIMES.active = True
    stream = torch.cuda.current_stream(device)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    t0.record(stream)
    for i in range(steps):
        fn(i)
    t1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    TIMES.active = False
    return t0.elapsed_time(t1), TIMES.summary(), clocks.stop()


def run_kv_microbench(args):
    """cached K/V bf16 N(0,1) [32 layers, 8 KV heads, 32768 tokens, 128]
    as 16 chunks x 2048 per layer; recomputed K = cached + N(0, 0.05) on a random 20 % of
    tokens; per-chunk RoPE target offsets uniform in [0, 32768); top-K at 10 %.  One step:
    assemble (all 32 layers, one launch) + HKVD per layer + fresh-row RoPE/scatter per layer."""
    import torch
    import cacheblend as cb
    from cacheblend import ops
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    L, Hkv, S, D, CL = args.kv_layers, args.kv_heads, 32768, 128, 2048
    Hq = 4 * Hkv
    n_chunks = S // CL
    kv = Hkv * D
    g = torch.Generator(device=device).manual_seed(0)
    cached_k = torch.randn((L, S, kv), generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    cached_v = torch.randn((L, S, kv), generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    sel = torch.rand((L, S, 1), generator=g, device=device) < 0.2
    k_new = (cached_k.float() + torch.randn((L, S, kv), generator=g, device=device) * 0.05 * sel).to(torch.bfloat16)
    del sel
    entries = [{"K": [cached_k[l, c * CL:(c + 1) * CL].unsqueeze(0) for l in range(L)],
                "V": [cached_v[l, c * CL:(c + 1) * CL].unsqueeze(0) for l in range(L)]} for c in range(n_chunks)]
    table = ops.ChunkTable(entries, range(L), device)
    deltas = torch.randint(0, 32768, (n_chunks,), generator=torch.Generator().manual_seed(1))
    positions = (deltas.repeat_interleave(CL) + torch.arange(CL).repeat(n_chunks)).to(device)
    invf = 1.0 / (1e6 ** (torch.arange(0, D, 2, dtype=torch.float32, device=device) / D))
    rope = ops.rope_table(invf, int(positions.max()) + 1)
    fk = torch.empty((L, S, kv), dtype=torch.bfloat16, device=device)
    fv = torch.empty_like(fk)
    k = ops.topk_count(S, 0.10)
    # fresh Q/K/V rows and the rotated Q per layer, as a model's projections give
    # them (one set for all layers would be read from L2 after the first)
    q_fresh = torch.randn((L, k, Hq * D), generator=g, device=device).to(torch.bfloat16)
    k_fresh = torch.randn((L, k, kv), generator=g, device=device).to(torch.bfloat16)
    v_fresh = torch.randn((L, k, kv), generator=g, device=device).to(torch.bfloat16)
    q_out = torch.empty((L, k, Hq * D), dtype=torch.bfloat16, device=device)
    rope_seq = ops.rope_table(invf, S)

    def step(i):
        ops.assemble_kv(table, 0, L, Hkv, D, rope, fk, fv, positions=positions)
        for l in range(L):
            # HKVD as its two kernels, so the HBM-bound deviation pass and the
            # latency-bound top-K select are timed apart
            dev = ops.kv_deviation_rows(k_new[l], table, l)
            idx = ops.topk_select(dev, k, force_last=True)
            ops.rope_scatter(q_fresh[l], k_fresh[l], v_fresh[l], idx, False, S, Hq, Hkv, D, rope_seq, fk[l],
                             fv[l], q_out=q_out[l])

    ms, kern, clk = _timed(step, args.steps, args.warmup, device)
    eager_ms = ms
    graph_note = None
    if not args.no_cuda_graph:
        # the same step captured once as a CUDA graph and replayed: 1 + 3L launches
        # with no Python between them (what BlendGraph does for a request)
        side = torch.cuda.Stream(device=device)
        side.wait_stream(torch.cuda.current_stream(device))
        step_graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            step(0)
            side.synchronize()
            with torch.cuda.graph(step_graph, stream=side):
                step(0)
        torch.cuda.current_stream(device).wait_stream(side)
        ms, _, clk = _timed(lambda i: step_graph.replay(), args.steps, args.warmup, device)
        del step_graph
        graph_note = "step captured once as a CUDA graph and replayed (eager launches from Python: eager_ms_per_step)"
    # Per-kernel rates: each kernel's L launches of one step captured once in a
    # CUDA graph and replayed between one CUDA-event pair, so the time is the
    # kernels' own (launched one by one from Python, a 20-30 us launch would
    # leave the device idle between these short kernels; a pair of events
    # around every launch would add its own latency).
    idx_l = [ops.topk_select(ops.kv_deviation_rows(k_new[l], table, l), k, force_last=True) for l in range(L)]
    devs = [ops.kv_deviation_rows(k_new[l], table, l) for l in range(L)]
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(device)

    def batch_ms(fn, reps):
        fn()
        side = torch.cuda.Stream(device=device)
        side.wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            fn()
            side.synchronize()
            with torch.cuda.graph(graph, stream=side):
                fn()
        stream.wait_stream(side)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) / reps

    per_kernel = {
        "assemble_kv": batch_ms(lambda: ops.assemble_kv(table, 0, L, Hkv, D, rope, fk, fv, positions=positions),
                                args.steps),
        "kv_deviation": batch_ms(lambda: [ops.kv_deviation_rows(k_new[l], table, l) for l in range(L)],
                                 args.steps),
        "topk_select": batch_ms(lambda: [ops.topk_select(devs[l], k, force_last=True) for l in range(L)],
                                args.steps),
        "rope_scatter": batch_ms(lambda: [ops.rope_scatter(q_fresh[l], k_fresh[l], v_fresh[l], idx_l[l], False,
                                                           S, Hq, Hkv, D, rope_seq, fk[l], fv[l], q_out=q_out[l])
                                          for l in range(L)], args.steps),
    }
    hbm, _, _, src = load_peaks()
    asm_b = L * 4 * S * kv * 2
    hk_b = L * (2 * S * kv * 2 + 4 * S)
    sc_b = L * k * (Hq * D + 2 * kv) * 2 * 2
    out = {}
    for name, nbytes in (("assemble_kv", asm_b), ("kv_deviation", hk_b), ("rope_scatter", sc_b)):
        n, t = kern.get(name, (0, 0.0))
        per_step = per_kernel[name]
        out[name] = {"launches_per_step": n // args.steps, "ms_per_step": round(per_step, 4),
                     "bytes_per_step": nbytes, "GB/s": round(nbytes / (per_step * 1e-3) / 1e9, 1),
                     "frac_hbm": round(nbytes / (per_step * 1e-3) / 1e9 / hbm, 3),
                     "ms_per_step_in_step_spans": round(t / args.steps, 4)}
    n_tk, _ = kern.get("topk_select", (0, 0.0))
    out["topk_select"] = {"launches_per_step": n_tk // args.steps, "bound": "latency (one CTA, S keys)",
                          "us_per_launch": round(per_kernel["topk_select"] / max(n_tk // args.steps, 1) * 1e3, 1)}
    total_b = asm_b + hk_b + sc_b
    print(json.dumps({
        "metric": "KV-kernel HBM GB/s (assemble + HKVD + scatter, microbench [32,8,32768,128])",
        "value": round(total_b / (ms / args.steps * 1e-3) / 1e9, 1), "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
        "eager_ms_per_step": round(eager_ms / args.steps, 3), "launch": graph_note or "eager",
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "kv-microbench", "layers": L, "kv_heads": Hkv, "tokens": S, "head_dim": D,
                   "chunks": f"{n_chunks}x{CL}", "topk": k,
                   "l2": f"inputs larger than L2 ({4 * L * S * kv / 1e9:.1f} GB chunk K/V; recomputed K, fresh Q/K/V rows and fused K/V per layer)"},
        "kernels": out, "hbm_peak_gbs": hbm, "hbm_peak_kind": src, "clocks": clk}), flush=True)


def run_decode_kernels(args):
    """One decode step's kernels at Mistral-7B shapes (7K blended cache), each
    timed as a CUDA-graph replay of a batch of launches over distinct buffers
    larger than L2: decode_attn over 32 layer caches of 6240 rows at position
    6208, and the one-row GEMVs of a layer (stacked q/k/v, o, stacked gate/up,
    down with the SiLU * up input) over 4 layers' weights, plus lm_head."""
    import torch
    from cacheblend import ops
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    H, I, Hq, Hkv, D, V = 4096, 14336, 32, 8, 128, 32000
    L, cap, p, NL = 32, 6240, 6208, 4
    bf = torch.bfloat16
    g = torch.Generator(device=device).manual_seed(0)

    def rnd(shape, scale=1.0):
        return (torch.randn(shape, generator=g, device=device) * scale).to(bf)

    kc = torch.stack([rnd((cap, Hkv * D)) for _ in range(L)])
    vc = torch.stack([rnd((cap, Hkv * D)) for _ in range(L)])
    q = rnd((Hq * D,))
    pos = torch.tensor([p], dtype=torch.int64, device=device)
    ws = ops.decode_workspace(cap, Hq, Hkv, D, device)
    ao = torch.empty((L, 1, Hq * D), dtype=bf, device=device)
    w_qkv = torch.stack([rnd((H + 2 * Hkv * D, H), 0.02) for _ in range(NL)])
    w_o = torch.stack([rnd((H, H), 0.02) for _ in range(NL)])
    w_gu = torch.stack([rnd((2 * I, H), 0.02) for _ in range(NL)])
    w_down = torch.stack([rnd((H, I), 0.02) for _ in range(NL)])
    w_lm = rnd((V, H), 0.02)
    x = rnd((1, 1, H))
    gu = rnd((1, 1, 2 * I), 3.0)
    stream = torch.cuda.current_stream(device)

    def graph_ms(fn, n_calls, reps):
        fn()
        side = torch.cuda.Stream(device=device)
        side.wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            fn()
            side.synchronize()
            with torch.cuda.graph(graph, stream=side):
                fn()
        stream.wait_stream(side)
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) / reps / n_calls

    kernels = {
        "decode_attn": (lambda: [ops.decode_attn(q, kc[l], vc[l], pos, Hq, Hkv, D, D ** -0.5, ws, out=ao[l])
                                 for l in range(L)], L, 2 * (p + 1) * Hkv * D * 2),
        "gemv_qkv": (lambda: [ops.gemv(w_qkv[l], x) for l in range(NL)], NL, w_qkv[0].numel() * 2),
        "gemv_o": (lambda: [ops.gemv(w_o[l], x) for l in range(NL)], NL, w_o[0].numel() * 2),
        "gemv_gate_up": (lambda: [ops.gemv(w_gu[l], x) for l in range(NL)], NL, w_gu[0].numel() * 2),
        # the GEMV forming SiLU * up while it stages its input (cbk_gemv's gate/up form)
        "gemv_down_silu": (lambda: [ops.gemv(w_down[l], gate=gu[..., :I], up=gu[..., I:]) for l in range(NL)],
                           NL, w_down[0].numel() * 2),
        "gemv_lm_head": (lambda: [ops.gemv(w_lm, x)], 1, w_lm.numel() * 2),
        # the decode step's down projection: one silu_mul launch, then the plain GEMV
        "silu_mul_then_gemv_down": (lambda: [ops.gemv(w_down[l], ops.silu_mul(gu[..., :I], gu[..., I:]))
                                             for l in range(NL)], NL, w_down[0].numel() * 2),
    }
    clocks = Clocks(0)
    clocks.start()
    time.sleep(0.3)
    hbm = load_peaks()[0]
    out, per_token_ms, per_token_bytes = {}, 0.0, 0
    for name, (fn, n, nbytes) in kernels.items():
        ms = graph_ms(fn, n, args.steps)
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"us_per_call": round(ms * 1e3, 2), "bytes_per_call": nbytes, "GB/s": round(gbs, 1),
                     "frac_hbm": round(gbs / hbm, 3)}
        if name == "gemv_down_silu":               # the alternative the decode step does not use
            continue
        calls = 1 if name == "gemv_lm_head" else 32
        per_token_ms += ms * calls
        per_token_bytes += nbytes * calls
    clk = clocks.stop()
    print(json.dumps({
        "metric": "decode-step kernels HBM GB/s (Mistral-7B, 7K blended cache)",
        "value": round(per_token_bytes / (per_token_ms * 1e-3) / 1e9, 1), "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_token_kernels": round(per_token_ms, 3),
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "decode-kernels", "cache_rows": cap, "position": p, "layers_timed": {"attention": L,
                   "gemv": NL}, "per_token": "32 x (attention + 4 GEMV) + lm_head",
                   "l2": "distinct buffers per launch in a batch (K/V 0.8 GB, weights 1.7 GB); lm_head 262 MB alone"},
        "kernels": out, "hbm_peak_gbs": hbm, "clocks": clk}), flush=True)


LLAMA3_8B = dict(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                 num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=5e5,
                 rms_norm_eps=1e-5, max_position_embeddings=131072)
L8_CHUNKS, L8_CHUNK_LEN, L8_QUERY_LEN, L8_RATIO, L8_REQUESTS = 16, 2048, 128, 0.10, 64


def run_llama8b_32k(args):
    """Llama-3-8B-shaped 32K blended prefill, 64 independent requests split by
    request over the ranks (no collective on the data path).  One step = every
    rank runs its 64/N requests through fuse_selective; the total work is the
    same 64 requests whatever N is: strong scaling.  Each rank keeps at most
    --requests distinct stored requests (their chunk KV is 4.3 GB each) and
    cycles through them."""
    import torch
    import torch.distributed as dist
    import cacheblend as cb
    from cacheblend._timing import TIMES
    from transformers import LlamaConfig, LlamaForCausalLM

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    if L8_REQUESTS % world:
        raise SystemExit(f"{L8_REQUESTS} requests do not split over {world} ranks")
    per_rank = L8_REQUESTS // world
    n_distinct = max(1, min(per_rank, args.requests if args.requests > 1 else 8))
    cfg = LlamaConfig(**LLAMA3_8B)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    with torch.device(device):
        model = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    lw = cb.LayerwiseModel.from_hf(model)
    store = cb.KVStore()
    reqs, ids = [], []
    for r in range(n_distinct):
        gen = torch.Generator().manual_seed(50_000 + 1000 * rank + r)
        lens = [L8_CHUNK_LEN] * L8_CHUNKS + [L8_QUERY_LEN]
        toks = [torch.randint(0, cfg.vocab_size, (n,), generator=gen).tolist() for n in lens]
        chunks = [cb.Chunk(text=f"l8r{rank}q{r}c{i}", token_ids=t,
                           chunk_id=cb.chunker._stable_id(f"l8r{rank}q{r}c{i}", t)) for i, t in enumerate(toks)]
        for c in chunks:
            K, V = cb.precompute_chunk_kv(lw, c)
            store.put(c.chunk_id, K, V)
        reqs.append(chunks)
        ids.append(torch.tensor([t for c in chunks for t in c.token_ids], dtype=torch.int64))
    S = sum(c.length for c in reqs[0])
    dev_ids = [t.to(device) for t in ids]
    pinned = [t.pin_memory() for t in ids]
    stream = torch.cuda.current_stream(device)

    def one(i, src, graph=True):
        # only the first token is needed: lm_head on the last position (the dense
        # (1, S, vocab) logits would be 8.4 GB per request)
        logits = cb.fuse_selective(lw, reqs[i % n_distinct], store, recompute_ratio=L8_RATIO,
                                   check_layer=CHECK_LAYER, input_ids=src[i % n_distinct], logits_rows="last",
                                   cuda_graph=None if graph else False)
        return logits[0, -1].argmax()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        for i in range(per_rank):
            one(i, dev_ids)
    torch.cuda.synchronize()
    clocks = Clocks(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        for i in range(per_rank):
            one(i, dev_ids)
    t1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(t0.elapsed_time(t1)) / args.steps
    # end to end: host ids in (pinned), first token out, per request
    barrier()
    torch.cuda.synchronize()
    a = time.perf_counter()
    for i in range(per_rank):
        int(one(i, pinned).item())
    e2e_ms = max_over_ranks((time.perf_counter() - a) * 1e3)
    # per-kernel device times inside the graph: a second capture of the request
    # geometry with external CUDA events around every libcbk launch, read after
    # each replay (one step's requests)
    TIMES.reset()
    TIMES.active = True
    tg = cb.BlendGraph(lw, reqs[0], store, recompute_ratio=L8_RATIO, check_layer=CHECK_LAYER,
                       logits_rows="last", dense_logits=False)
    TIMES.active = False
    spans = list(TIMES.graph_spans)
    TIMES.reset()
    acc = {}
    for i in range(per_rank):
        tg.replay(reqs[i % n_distinct], store, input_ids=dev_ids[i % n_distinct])
        torch.cuda.synchronize()
        TIMES.read_graph_spans(spans, acc)
    del tg
    kern = {name: (v[0], v[1]) for name, v in acc.items()}
    launches = sum(v[2] for v in acc.values()) * args.steps
    n_sp, ms_sp = kern.get("partial_attn", (0, 0.0))
    _, idx = cb.fuse_selective(lw, reqs[0], store, recompute_ratio=L8_RATIO, check_layer=CHECK_LAYER,
                               return_hkvd_indices=True)
    sel = sum(int(p) + 1 for p in idx.cpu().tolist())
    fl_sp = 4 * cfg.num_attention_heads * cfg.head_dim * sel
    hbm_peak, tf_burst, tf_sust, peak_src = load_peaks()
    tf_sp = fl_sp / (ms_sp / n_sp * 1e-3) / 1e12 if n_sp else None
    res = {
        "metric": "blended-prefill requests/s (Llama-3-8B shape, 32K ctx, 64 requests)",
        "value": round(L8_REQUESTS / (ms * 1e-3), 3), "unit": "requests/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 1),
        "ttft_ms_per_request": round(ms / per_rank, 2), "tokens_per_s": round(L8_REQUESTS * S / (ms * 1e-3), 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform-random token ids; random-init weights)",
        "config": {"workload": "llama3-8b-32k-x64", "model": "Llama-3-8B architecture, random init",
                   "chunks": f"{L8_CHUNKS}x{L8_CHUNK_LEN}+{L8_QUERY_LEN}", "S": S, "recompute_ratio": L8_RATIO,
                   "k_selected": int(idx.numel()), "check_layer": CHECK_LAYER, "requests": L8_REQUESTS,
                   "requests_per_rank": per_rank, "distinct_requests_per_rank": n_distinct,
                   "parallelism": f"by-request x{world}", "logits_rows": "last",
                   "l2": "inputs larger than L2 (16 GB weights, 4.3 GB fused KV per request)"},
        "e2e": {"value": round(L8_REQUESTS / (e2e_ms * 1e-3), 3), "unit": "requests/s",
                "ms_per_step": round(e2e_ms, 1), "h2d_bytes_per_step": per_rank * S * 8,
                "d2h_bytes_per_step": per_rank * 8},
        "roofline": {"kernel": "partial_attn_kernel", "bound": "tensor",
                     "achieved": round(tf_sp, 1) if tf_sp else None, "peak": tf_sust, "unit": "TFLOP/s",
                     "frac": round(tf_sp / tf_sust, 4) if tf_sp else None, "peak_kind": f"{peak_src} bf16 sustained",
                     "flops_per_launch": fl_sp, "calls": n_sp, "avg_launch_ms": round(ms_sp / max(n_sp, 1), 4)},
        "kernels": {k: {"calls": v[0], "avg_ms": round(v[1] / max(v[0], 1), 4)} for k, v in kern.items()},
        "gpu_launches": launches,
        "clocks": clk,
    }
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


LLAMA3_70B = dict(layers=80, n_q=64, n_kv=8, head_dim=128, theta=5e5)
SH_CHUNKS, SH_CHUNK_LEN, SH_QUERY_LEN, SH_RATIO = 64, 2048, 256, 0.15


def run_kv_sharded(args):
    """Llama-3-70B-shaped 128K blended prefill hot path, KV heads sharded over
    the ranks (rank r keeps KV heads [r*8/N, (r+1)*8/N) and their q heads).
    Per step: (a)+(b) assemble of every cached layer, the dense layer before the
    check layer (fresh rows for all tokens), (c) HKVD: partial deviation over
    this rank's heads, NCCL all-gather of the S fp32 partials, the same top-K
    on every rank, then per sparse layer (b)+(d) RoPE + scatter of the fresh
    rows and (e) partial attention.  Projections / MLP would need tensor-parallel
    all-reduces and are not on this path: the fresh Q/K/V rows are seeded
    synthetic inputs (one set reused by every layer).  Total work is one request
    whatever N is: strong scaling."""
    import torch
    import torch.distributed as dist
    from cacheblend import ops
    from cacheblend._timing import TIMES
    from cacheblend.sharding import head_shard, sharded_hkvd_select

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    c = LLAMA3_70B
    L, Hq, Hkv, D = args.sh_layers, c["n_q"], c["n_kv"], c["head_dim"]
    ck = CHECK_LAYER
    lo, hi = head_shard(Hkv, world, rank)
    hkv = hi - lo
    hq = hkv * (Hq // Hkv)
    kvd = hkv * D
    lens = [SH_CHUNK_LEN] * SH_CHUNKS + [SH_QUERY_LEN]
    S = sum(lens)
    k_sel = max(1, min(S, int(S * SH_RATIO)))
    bf = torch.bfloat16

    def randn(shape, seed):
        g = torch.Generator(device=device).manual_seed(seed)
        return torch.randn(shape, generator=g, device=device, dtype=torch.float32).to(bf)

    def heads(seed_of, h_lo, h_hi):
        """(S, (h_hi - h_lo) * D) bf16: KV head h's columns seeded by seed_of(h), so the
        whole-model data (and the selection) is the same for every rank count"""
        return torch.cat([randn((S, D), seed_of(h)) for h in range(h_lo, h_hi)], dim=1)

    # per-layer chunk K/V of this rank's heads (chunks are row ranges of one buffer)
    ck_k = [heads(lambda h, l=l: 1_000_000 * h + 2 * l, lo, hi) for l in range(L)]
    ck_v = [heads(lambda h, l=l: 1_000_000 * h + 2 * l + 1, lo, hi) for l in range(L)]
    starts = [0]
    for n in lens:
        starts.append(starts[-1] + n)
    entries = [{"K": [ck_k[l][a:b].unsqueeze(0) for l in range(L)],
                "V": [ck_v[l][a:b].unsqueeze(0) for l in range(L)]} for a, b in zip(starts, starts[1:])]
    table = ops.ChunkTable(entries, range(ck, L), device)
    inv_freq = 1.0 / (c["theta"] ** (torch.arange(0, D, 2, dtype=torch.float32, device=device) / D))
    rope = ops.rope_table(inv_freq, S)
    fused_k = torch.empty((L, S, kvd), dtype=bf, device=device)
    fused_v = torch.empty_like(fused_k)
    # recomputed check-layer K = cached + N(0, 0.05) on a random 20% of tokens
    # (the token mask is common to all ranks: the same tokens are recomputed)
    gm = torch.Generator(device=device).manual_seed(77)
    mask = (torch.rand((S, 1), generator=gm, device=device) < 0.2).float()
    noise_seed = lambda h: 1_000_000 * h + 999_999
    k_fresh = (ck_k[ck].float() + heads(noise_seed, lo, hi).float() * 0.05 * mask).to(bf)
    q_all, k_all, v_all = randn((S, hq * D), 5 + rank), randn((S, kvd), 6 + rank), randn((S, kvd), 7 + rank)
    q_rows, k_rows, v_rows = q_all[:k_sel], k_all[:k_sel], v_all[:k_sel]
    pos_all = torch.arange(S, device=device, dtype=torch.int64)
    scale = D ** -0.5
    ws_dense = ops.attn_workspace(S, S, hq, hkv, D, device)
    ws_sparse = ops.attn_workspace(k_sel, S, hq, hkv, D, device)
    q_dense = torch.empty((S, hq * D), dtype=bf, device=device)
    q_sparse = torch.empty((k_sel, hq * D), dtype=bf, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device)

    def step(k_check):
        ops.assemble_kv(table, ck, L, hkv, D, rope, fused_k, fused_v, status=status)
        for li in range(ck):
            ops.rope_scatter(q_all, k_all, v_all, pos_all, False, S, hq, hkv, D, rope, fused_k[li],
                             fused_v[li], q_out=q_dense, status=status)
            ops.partial_attn(q_dense, fused_k[li], fused_v[li], pos_all, hq, hkv, D, scale, status=status,
                             workspace=ws_dense, reuse_plan=li > 0, timer_tag="_dense")
        idx = sharded_hkvd_select(k_check, table, ck, k_sel)
        for li in range(ck, L):
            if li == ck:      # check layer: fresh rows gathered from the full-row projections
                ops.rope_scatter(q_all, k_check, v_all, idx, True, S, hq, hkv, D, rope, fused_k[li],
                                 fused_v[li], q_out=q_sparse, status=status)
            else:
                ops.rope_scatter(q_rows, k_rows, v_rows, idx, False, S, hq, hkv, D, rope, fused_k[li],
                                 fused_v[li], q_out=q_sparse, status=status)
            ops.partial_attn(q_sparse, fused_k[li], fused_v[li], idx, hq, hkv, D, scale, status=status,
                             workspace=ws_sparse, reuse_plan=li > ck)
        return idx

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        idx = step(k_fresh)
    torch.cuda.synchronize()
    # every rank must hold the identical selection ...
    same = True
    if world > 1:
        allidx = torch.empty((world, k_sel), dtype=torch.int64, device=device)
        dist.all_gather_into_tensor(allidx, idx)
        same = bool((allidx == allidx[0:1]).all().item())
    # ... and it must be the selection one GPU makes from all heads: rank 0 rebuilds
    # the check layer's fresh and cached K of every head and runs the unsharded HKVD
    single = None
    if rank == 0:
        k_old_all = heads(lambda h: 1_000_000 * h + 2 * ck, 0, Hkv)
        k_new_all = (k_old_all.float() + heads(noise_seed, 0, Hkv).float() * 0.05 * mask).to(bf)
        ent_all = [{"K": [k_old_all[a:b].unsqueeze(0)], "V": [k_old_all[a:b].unsqueeze(0)]}
                   for a, b in zip(starts, starts[1:])]
        dev_all = ops.kv_deviation_rows(k_new_all, ops.ChunkTable(ent_all, [0], device), 0)
        single = bool(torch.equal(ops.topk_select(dev_all, k_sel, force_last=True), idx))
        del k_old_all, k_new_all, ent_all, dev_all
    del mask
    sel_digest = int(torch.sum(idx * torch.arange(1, k_sel + 1, device=device)).item())

    clocks = Clocks(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    TIMES.reset()
    TIMES.active = True
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        idx = step(k_fresh)
    t1.record(stream)
    torch.cuda.synchronize()
    TIMES.active = False
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(t0.elapsed_time(t1)) / args.steps
    kern = TIMES.summary()
    launches = sum(TIMES.launches.values())

    # end to end: the check-layer K from pinned host memory, the selection back to the host
    k_host = k_fresh.cpu().pin_memory()
    k_dev = torch.empty_like(k_fresh)
    barrier()
    torch.cuda.synchronize()
    e2e = []
    for _ in range(args.steps):
        a = time.perf_counter()
        k_dev.copy_(k_host, non_blocking=True)
        idx_host = step(k_dev).cpu()
        e2e.append((time.perf_counter() - a) * 1e3)
    barrier()
    e2e_ms = max_over_ranks(sum(e2e) / len(e2e))
    st = int(status.item())

    idx_l = idx_host.tolist()
    sel = sum(int(p) + 1 for p in idx_l)
    fl_sp = 4 * hq * D * sel
    fl_de = 4 * hq * D * (S * (S + 1) // 2)
    n_sp, ms_sp = kern.get("partial_attn", (0, 0.0))
    n_de, ms_de = kern.get("partial_attn_dense", (0, 0.0))
    n_asm, asm_ms = kern.get("assemble_kv", (0, 0.0))
    asm_bytes = (L - ck) * 2 * 2 * S * kvd * 2
    hbm_peak, tf_burst, tf_sust, peak_src = load_peaks()
    tf_sp = fl_sp / (ms_sp / n_sp * 1e-3) / 1e12 if n_sp else None
    res = {
        "metric": "KV-head-sharded blended-prefill hot path tokens/s (Llama-3-70B shape, 128K ctx)",
        "value": round(S / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) chunk K/V and fresh rows; recomputed K = cached + N(0,0.05) on 20%)",
        "config": {"workload": "llama70b-128k-sharded", "layers": L, "S": S, "k_selected": k_sel,
                   "chunks": f"{SH_CHUNKS}x{SH_CHUNK_LEN}+{SH_QUERY_LEN}", "q_heads_per_rank": hq,
                   "kv_heads_per_rank": hkv, "head_dim": D, "check_layer": ck,
                   "parallelism": f"kv-heads/{world}",
                   "exchange": "NCCL all_gather of S fp32 partials, combined by the deviation's pairwise tree",
                   "selection_identical_on_all_ranks": same, "selection_equals_single_gpu": single,
                   "selection_digest": sel_digest, "status": st,
                   "l2": "inputs larger than L2 (per-layer K/V buffers)"},
        "e2e": {"value": round(S / (e2e_ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(e2e_ms, 3),
                "h2d_bytes_per_step": S * kvd * 2, "d2h_bytes_per_step": k_sel * 8},
        "roofline": {"kernel": "partial_attn_kernel", "bound": "tensor",
                     "achieved": round(tf_sp, 1) if tf_sp else None, "peak": tf_sust, "unit": "TFLOP/s",
                     "frac": round(tf_sp / tf_sust, 4) if tf_sp else None,
                     "peak_kind": f"{peak_src} bf16 sustained", "flops_per_launch": fl_sp, "calls": n_sp,
                     "avg_launch_ms": round(ms_sp / max(n_sp, 1), 4)},
        "kernels": {
            "assemble_kv": {"calls": n_asm, "avg_ms": round(asm_ms / max(n_asm, 1), 3), "bytes": asm_bytes,
                            "GB/s": round(asm_bytes / (asm_ms / n_asm * 1e-3) / 1e9, 1) if n_asm else None},
            "partial_attn_dense": {"calls": n_de, "avg_ms": round(ms_de / max(n_de, 1), 3),
                                   "TFLOP/s": round(fl_de / (ms_de / n_de * 1e-3) / 1e12, 1) if n_de else None},
            "hkvd_partial_plus_exchange": {k: round(v[1] / max(v[0], 1), 4) for k, v in kern.items()
                                           if k in ("kv_deviation", "topk_select")},
        },
        "gpu_launches": launches,
        "clocks": clk,
    }
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


def run_decode(args):
    """Mistral-7B 7K blend followed by greedy decode over the blended cache
    (generate_greedy): ms per decoded token after the prefill, device time."""
    import torch
    import cacheblend as cb
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    model = build_model(device)
    lw = cb.LayerwiseModel.from_hf(model)
    store = cb.KVStore()
    chunks = build_request(model, cb, seed=0, device=device)
    for c in chunks:
        K, V = cb.precompute_chunk_kv(lw, c)
        store.put(c.chunk_id, K, V)
    n_new = args.decode_tokens
    for _ in range(args.warmup):
        cb.generate_greedy(lw, chunks, store, 2, recompute_ratio=RATIO, check_layer=CHECK_LAYER)
    torch.cuda.synchronize()
    res = []
    for n in (1, n_new):
        t0 = time.perf_counter()
        for _ in range(args.steps):
            toks = cb.generate_greedy(lw, chunks, store, n, recompute_ratio=RATIO, check_layer=CHECK_LAYER)
        torch.cuda.synchronize()
        res.append((time.perf_counter() - t0) * 1e3 / args.steps)
    per_tok = (res[1] - res[0]) / (n_new - 1)
    # the reference's decode on the same blended cache: HF forward with past_key_values
    with torch.inference_mode():
        out = cb.fuse_selective(lw, chunks, store, recompute_ratio=RATIO, check_layer=CHECK_LAYER,
                                return_layerwise_output=True)
        cache, nxt = out.past_key_values, out.logits[0, -1].argmax().view(1, 1)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(n_new - 1):
            step = model(input_ids=nxt, past_key_values=cache, use_cache=True)
            cache, nxt = step.past_key_values, step.logits[0, -1].argmax().view(1, 1)
            int(nxt.item())
        torch.cuda.synchronize()
        hf_per_tok = (time.perf_counter() - t0) * 1e3 / (n_new - 1)
    print(json.dumps({
        "metric": "greedy decode over the blended cache, ms per token (Mistral-7B 7K blend)",
        "value": round(per_tok, 3), "unit": "ms/token", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": False, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "mistral7b-7k-decode", "S": sum(c.length for c in chunks), "new_tokens": n_new,
                   "prefill_plus_first_token_ms": round(res[0], 2), "tokens": toks[:8]},
        "hf_decode_ms_per_token": round(hf_per_tok, 3),
        "note": "host wall time per call (each token is read back to choose the next, as in the reference)"}),
        flush=True)


def run_attn_layers(args):
    """Partial attention alone at the Mistral-7B sparse-layer shape: S = 6208 keys,
    k = 931 selected rows (uniform random, last position included), 32 q / 8 KV heads,
    D = 128; 31 distinct layer buffers (0.8 GB, larger than L2) cycled per launch."""
    import torch
    from cacheblend import ops
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    S, k, Hq, Hkv, D, L = 6208, min(args.attn_k, 6208), 32, 8, 128, args.attn_layers
    g = torch.Generator(device=device).manual_seed(0)
    gc = torch.Generator().manual_seed(0)
    if k == S:
        pos = torch.arange(S, device=device)
    elif args.attn_dist == "tail":      # the last k positions (a selection clustered at the end)
        pos = torch.arange(S - k, S, device=device)
    elif args.attn_dist == "blend":     # like the 7K blend's HKVD picks: none in chunk 0 (its K equals
        # the cached K), 37 % in the last 1088 positions, the rest uniform over [1024, 5120)
        n_tail = int(0.373 * k) - 1
        tail = torch.randperm(S - 1 - 5120, generator=gc)[:n_tail] + 5120
        mid = torch.randperm(5120 - 1024, generator=gc)[:k - 1 - n_tail] + 1024
        pos = torch.cat([torch.sort(torch.cat([mid, tail])).values, torch.tensor([S - 1])]).to(device)
    else:
        pos = torch.cat([torch.sort(torch.randperm(S - 1, generator=gc)[:k - 1]).values,
                         torch.tensor([S - 1])]).to(device)
    kc = torch.randn((L, S, Hkv * D), generator=g, device=device).to(torch.bfloat16)
    vc = torch.randn((L, S, Hkv * D), generator=g, device=device).to(torch.bfloat16)
    q = torch.randn((L, k, Hq * D), generator=g, device=device).to(torch.bfloat16)
    out = torch.empty((k, Hq * D), dtype=torch.bfloat16, device=device)
    ws = ops.attn_workspace(k, S, Hq, Hkv, D, device)

    def step(i):
        for l in range(L):   # one plan per step, reused by the other layers (as in fuse_selective)
            ops.partial_attn(q[l], kc[l], vc[l], pos, Hq, Hkv, D, D ** -0.5, out=out, workspace=ws,
                             reuse_plan=l > 0)

    ms, kern, clk = _timed(step, args.steps, args.warmup, device)
    n, t = kern["partial_attn"]
    flops = attn_flops(pos.tolist(), S, Hq, D, 0, 1)
    _, _, tf_sust, src = load_peaks()
    _, tf_burst, _, _ = load_peaks()
    ach = flops / (t / n * 1e-3) / 1e12
    print(json.dumps({
        "metric": "partial attention TFLOP/s (Mistral-7B sparse layer)", "value": round(ach, 1),
        "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic", "config": {"workload": "attn-layers", "S": S, "k": k, "layers": L,
                                        "selection": args.attn_dist},
        "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": tf_burst, "unit": "TFLOP/s",
                     "frac": round(ach / tf_burst, 4), "peak_kind": f"{src} bf16 burst (kernel timed alone)",
                     "flops_per_launch": flops, "avg_launch_ms": round(t / n, 5)},
        "clocks": clk}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--requests", type=int, default=1, help="distinct requests per rank (cycled)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="mistral7b-7k-blend",
                    choices=["mistral7b-7k-blend", "kv-microbench", "attn-layers", "llama70b-128k-sharded",
                             "llama3-8b-32k-x64", "mistral7b-7k-decode", "decode-kernels"])
    ap.add_argument("--attn-layers", type=int, default=31)
    ap.add_argument("--attn-k", type=int, default=931, help="selected rows (6208 = dense causal)")
    ap.add_argument("--attn-dist", default="uniform", choices=["uniform", "tail", "blend"])
    ap.add_argument("--sh-layers", type=int, default=80, help="layers of the sharded 128K workload")
    ap.add_argument("--kv-layers", type=int, default=32, help="layers of the KV microbench")
    ap.add_argument("--kv-heads", type=int, default=8,
                    help="KV heads of the KV microbench (1: the rows one rank holds with 8 heads over 8 GPUs)")
    ap.add_argument("--kv-arena", action="store_true", help="chunk K/V in one KVArena device pool")
    ap.add_argument("--decode-tokens", type=int, default=32, help="tokens of the decode workload")
    ap.add_argument("--no-cuda-graph", action="store_true",
                    help="time fuse_selective(cuda_graph=False) (kernel by kernel) instead of the graph replay")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "kv-microbench":
        run_kv_microbench(args)
    elif args.workload == "attn-layers":
        run_attn_layers(args)
    elif args.workload == "llama70b-128k-sharded":
        run_kv_sharded(args)
    elif args.workload == "llama3-8b-32k-x64":
        run_llama8b_32k(args)
    elif args.workload == "mistral7b-7k-decode":
        run_decode(args)
    elif args.workload == "decode-kernels":
        run_decode_kernels(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
