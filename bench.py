"""Benchmark of the B200 decode backend (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|gemv_fp8] [--context 512] [--no-cpu]

Workload `decode` (default): batch-1 greedy decode of the
Flash-scale model -- 43 layers, hidden 4096, 256 FP4 routed experts (inter
2048, top-6) + 1 shared FP8 expert per layer, MLA with the lightning indexer,
vocab 129280 -- with random-init weights generated directly in HBM (≈157 GB,
every weight resident). A 512-token random prompt is run first (untimed,
token by token through the same captured step), then W untimed and K timed
decode steps. One step = one token = one replay of the captured CUDA graph;
steps are timed with CUDA events on the model's stream. Every step streams
≈11.1 GB of distinct weights, far more than the 126 MB L2, so no flush is
needed between steps. `value` is tokens/s of the sequence; `e2e` times the
reference-facing call dsv4_cuda_model_decode (host token and position in,
host next token out) with the host wall clock. Under torchrun the one
sequence is decoded by the model sharded over the N GPUs (expert inter
slices, q heads / o_groups, wo_b columns, LM-head vocabulary; two exchanges
per layer over NVLink peer memory), every rank stepping in lockstep (strong
scaling); the slowest rank's time is reported.

Workload `gemv_fp8`: y = W x with W 4096x7168 e4m3 in
128x128 E8M0 blocks, one GEMV per step over 8 rotating resident copies (235 MB
> L2), graph-launched; value in algorithmic HBM GB/s.

--impl reference times the reference's own CPU code (oracle/_ref, built from
its sources) on the host cores on the same workload: for `decode`, its
dsv4_layer_forward on a 3-layer Flash-geometry sample (one layer of each
compress ratio 0 / 4 / 128, all 256 experts, the full-vocab head), scaled to
the 43-layer mix; for `gemv_fp8`, dsv4_matmul_fp8.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "deepseek-v4-in-c_b200"))
sys.path.insert(0, os.path.join(REPO, "oracle"))

C1_ROWS, C1_COLS = 4096, 7168
# algorithmic bytes of one config-1 GEMV: W + S + x + y
C1_BYTES = C1_ROWS * C1_COLS + 32 * 56 + C1_COLS * 4 + C1_ROWS * 4
NCOPY = 8

DECODE_METRIC = "batch-1 decode tok/s (Flash-scale synthetic, config 5)"


def decode_metric(batch):
    return DECODE_METRIC if batch == 1 else "batch-%d decode tok/s (Flash-scale synthetic, config 5)" % batch


def expected_experts(d, batch):
    """Expected distinct routed experts of a layer when `batch` tokens each
    pick topk of n_experts uniformly: the experts a batched step must read."""
    E, K = d["n_experts"], d["topk"]
    return E * (1.0 - (1.0 - K / E) ** batch)


def decode_bytes_per_step(d, pos, batch):
    """Algorithmic HBM bytes of one batched step: the weights once (the routed
    experts as the expected distinct ones of the batch), every sequence's KV."""
    one = decode_bytes_per_token(d, pos)
    if batch == 1:
        return one
    per_expert = 3 * fp4_bytes(d["moe_inter"], d["hidden"])
    nl = len(layer_ratios(d))
    kv = decode_bytes_per_token(d, pos) - decode_bytes_per_token(d, 0)
    return one + nl * (expected_experts(d, batch) - d["topk"]) * per_expert + (batch - 1) * kv
GEMV_METRIC = "FP8 block-scaled GEMV HBM GB/s (config 1, 4096x7168 e4m3, batch 1)"


def prefill_metric(n_prompt, chunk):
    return ("prefill tok/s (Flash-scale synthetic, config 5, %d-token prompt in passes of %d)"
            % (n_prompt, chunk))


def prefill_bytes(d, n_prompt, chunk):
    """Algorithmic HBM bytes of a whole prefill: per pass every weight once
    (the routed experts as the expected distinct ones of the pass's tokens)
    and every token's attended KV rows; the LM head once (the prompt's last
    token only)."""
    head = d["vocab"] * d["hidden"] * 2
    per_expert = 3 * fp4_bytes(d["moe_inter"], d["hidden"])
    nl = len(layer_ratios(d))
    b0 = decode_bytes_per_token(d, 0)
    total = head
    for p0 in range(0, n_prompt, chunk):
        nt = min(chunk, n_prompt - p0)
        total += decode_bytes_per_token(d, p0) - head + nl * (expected_experts(d, nt) - d["topk"]) * per_expert
        total += sum(decode_bytes_per_token(d, p0 + t) - b0 for t in range(1, nt))
    return total

# DRAM bytes (read + write) per unit from an ncu capture of the same kernel
# and workload, or None where none was taken.
TRAFFIC_C1 = 29456384          # one config-1 GEMV launch (ncu dram__bytes_read + write)
# One decode token's DRAM bytes (read + write, every launch of the token) from
# an ncu capture at an early prompt position, and the algorithmic bytes of
# that position; a timed position adds the algorithmic difference (its KV rows).
TRAFFIC_DECODE = (11.2048e9, 11.1257e9)


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """SM clock, power and clock-event reasons of the bench's GPU, read through
    NVML every 100 ms by a thread while the timed region runs (read-only
    queries). The device is matched to the CUDA device by its UUID, so the
    sample is of the GPU the kernels run on whatever CUDA_VISIBLE_DEVICES
    maps. Falls back to one nvidia-smi query per sample."""
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))

    def __init__(self, dev):
        self.dev, self.rows, self.stop, self.err = dev, [], threading.Event(), None

    def _nvml(self):
        import pynvml as N
        import torch
        N.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.dev).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        h = N.nvmlDeviceGetHandleByUUID(uuid)
        mx = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)

        def one():
            return (N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM), mx,
                    N.nvmlDeviceGetPowerUsage(h) / 1000.0, N.nvmlDeviceGetCurrentClocksEventReasons(h))
        return one

    def _smi(self):
        q = "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active"

        def one():
            out = subprocess.run(["nvidia-smi", "-i", str(self.dev), "--query-gpu=" + q,
                                  "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                 timeout=5).stdout.strip().split(",")
            return float(out[0]), float(out[1]), float(out[2]), int(out[3].strip(), 16)
        return one

    def _run(self):
        try:
            try:
                one = self._nvml()
            except Exception as e:          # no NVML binding: the CLI
                self.err = "nvml: %s" % e
                one = self._smi()
            while True:
                self.rows.append(one())
                if self.stop.wait(0.1):
                    break
        except Exception as e:
            self.err = str(e)

    def __enter__(self):
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()
        time.sleep(0.15)                      # the first sample precedes the timed work
        return self

    def __exit__(self, *a):
        self.stop.set()
        self.t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled: %s" % self.err]}
        sm = [r[0] for r in self.rows]
        reasons = sorted({n for r in self.rows for n, bit in self.REASONS if r[3] & bit})
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(r[1] for r in self.rows)),
                "reasons": reasons, "power_w_max": round(max(r[2] for r in self.rows), 1),
                "samples": len(self.rows)}


def dist_setup(n):
    if n <= 1 or "RANK" not in os.environ:
        return 0, 1, None
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    os.environ["DSV4_DEVICE"] = str(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                            device_id=torch.device("cuda", local))
    return rank, world, dist


def max_over_ranks(dist, ms, device="cuda"):
    """The slowest rank's value (every rank calls it, in the same order)."""
    if not dist:
        return ms
    import torch
    t = torch.tensor([float(ms)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------ decode model

def flash_cfg():
    import dsv4_model as M
    return M.flash_config()


def layer_ratios(d):
    return list(d["compress_ratios"][:d["n_layers"]])


def fp8_bytes(rows, cols):
    return rows * cols + -(-rows // 128) * -(-cols // 128)


def fp4_bytes(rows, cols):
    return rows * cols // 2 + rows * cols // 32


def decode_bytes_per_token(d, pos):
    """Algorithmic HBM bytes of one batch-1 decode token at position pos: every
    weight the token reads once (trunk, router, the top-k routed and the
    shared experts, compressor / indexer weights, mHC, norms, LM head, the
    embedding row) plus the cached KV / key rows it attends over. Activations
    (< 1 MB) are left out."""
    hid, H, hd, ql = d["hidden"], d["n_heads"], d["head_dim"], d["q_lora"]
    og, ol, I, E, K = d["o_groups"], d["o_lora"], d["moe_inter"], d["n_experts"], d["topk"]
    hc, win = d["hc_mult"], d["sliding_window"]
    ih, idim, itop = d["index_n_heads"], d["index_head_dim"], d["index_topk"]
    mix = (2 + hc) * hc
    total = 0
    for r in layer_ratios(d):
        b = fp8_bytes(ql, hid) + fp8_bytes(H * hd, ql) + fp8_bytes(hd, hid)
        b += fp8_bytes(og * ol, H * hd // og) + fp8_bytes(hid, og * ol)
        b += 2 * mix * hc * hid * 4 + 2 * mix * 4 + 2 * 3 * 4          # mHC fn, base, scale
        b += (2 * hid + ql + hd + H) * 4                                # norms, sinks
        n_win = min(pos + 1, win)
        n_sel = 0
        if r:
            coff = 2 if r == 4 else 1
            b += 2 * (coff * hd * hid * 2) + coff * hd * 4 + hd * 4     # wkv / wgate bf16, ape row, norm
            n_comp = (pos + 1) // r
            n_sel = n_comp
            if r == 4:
                b += fp8_bytes(ih * idim, ql) + ih * hid * 2            # indexer wq_b, weights_proj
                b += n_comp * idim * 4                                  # indexer keys
                n_sel = min(n_comp, itop)
        b += (n_win + n_sel) * hd * 4                                   # attended KV rows (f32)
        b += E * hid * 2 + E * 4                                        # router bf16, bias
        b += K * (2 * fp4_bytes(I, hid) + fp4_bytes(hid, I))           # routed experts
        b += 2 * fp8_bytes(I, hid) + fp8_bytes(hid, I)                 # shared expert
        total += b
    total += hc * hc * hid * 4 + hid * 4 + d["vocab"] * hid * 2 + hid * 2  # hc_head, norm, head, embed row
    return total


def cpu_decode_sample(n_pos, warm=2, prompt_len=0):
    """The reference's dsv4_layer_forward on a 3-layer Flash-geometry model
    (compress ratios 0 / 4 / 128, all 256 experts, vocab 129280): without a
    prompt, n_pos positions after `warm` from a one-token prompt; with
    prompt_len, the GPU arm's random prompt of that length first (untimed),
    then `warm` and n_pos timed greedy positions, i.e. positions prompt_len +
    warm .. prompt_len + warm + n_pos - 1. Returns (seconds per 43-layer
    token, per-position times, description, first timed position)."""
    import oracle as O
    import dsv4_model as M
    full = layer_ratios(M.flash_config())
    count = {r: full.count(r) for r in set(full)}
    d = M.flash_sample_config()
    t0 = time.perf_counter()
    sm = M.SyntheticModel(d, seed=0, fast=True)
    t_build = time.perf_counter() - t0
    t0 = time.perf_counter()
    if prompt_len:
        prompt = np.random.default_rng(0).integers(0, d["vocab"], prompt_len).astype(np.int32)
        tl, th, _ = O.model_decode_timed_ref(sm, n_pos + warm, prompt=prompt)
        first = prompt_len + warm
    else:
        tl, th, _ = O.model_decode_timed_ref(sm, n_pos + warm)
        first = warm
    t_run = time.perf_counter() - t0
    tl, th = tl[first:first + n_pos], th[first:first + n_pos]
    per = tl[:, 0] * count[0] + tl[:, 1] * count[4] + tl[:, 2] * count[128] + th
    desc = ("reference dsv4_layer_forward + hc_head/norm/LM head/argmax (oracle/_ref) on a 3-layer "
            "Flash-geometry sample (ratios 0/4/128, 256 experts, vocab 129280), positions %d..%d%s, "
            "per-layer times scaled to the 43-layer mix (%d/%d/%d); OMP_NUM_THREADS=%s; sample build "
            "%.0f s, run %.0f s"
            % (first, first + n_pos - 1,
               " after the GPU arm's %d-token prompt (untimed)" % prompt_len if prompt_len
               else " after %d warm-up from position 0" % warm,
               count[0], count[4], count[128],
               os.environ.get("OMP_NUM_THREADS", "all %d" % os.cpu_count()), t_build, t_run))
    return float(np.sum(per) / n_pos), per, desc, first


def run_decode(a):
    import torch
    import dsv4_b200 as B
    import dsv4_model as M
    rank, world, dist = dist_setup(a.gpus)
    L = B.init()
    d = M.flash_config()
    W, K, P = max(a.warmup, 3), a.steps, a.context
    NB = a.batch
    if NB > 1 and world > 1:
        raise SystemExit("--batch > 1 runs on one GPU")
    n_e2e = max(16, min(K, 128))
    max_pos = P + W + K + n_e2e + 8
    cfg = M.ConfigOnly(d)
    t0 = time.perf_counter()
    if NB > 1:
        model = B.Model(cfg, max_pos, synthetic_seed=1234, n_seq=NB)
    elif world > 1:
        # one model sharded over the ranks: experts by inter slice, heads and
        # o_groups, wo_b columns, the LM head's vocabulary (NCCL exchanges)
        nid = [B.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(nid, src=0)
        model = B.Model(cfg, max_pos, synthetic_seed=1234, rank=rank, world=world, nccl_id=nid[0])
    else:
        model = B.Model(cfg, max_pos, synthetic_seed=1234)
    t_create = time.perf_counter() - t0
    resident = model.device_bytes()
    prompt = np.random.default_rng(0).integers(0, d["vocab"], P).astype(np.int32)
    if NB > 1:
        # sequence 0 takes the batch-1 prompt, the others their own
        rest = np.random.default_rng(1).integers(0, d["vocab"], (NB - 1, P)).astype(np.int32)
        model.begin_batch(np.concatenate([prompt[None, :], rest]))
    else:
        model.begin(prompt)
    launches_per_step = L.dsv4_cuda_model_step_kernels(model.h)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream

    def replay(n):
        for _ in range(n):
            B.check(L.dsv4b_model_step_async(model.h, sp), "dsv4b_model_step_async")

    replay(P)                  # the prompt, token by token (untimed)
    replay(W)                  # warm-up decode steps
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(torch.cuda.current_device()) as clk:
        torch.cuda.synchronize()
        e0.record(stream)
        replay(K)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = max_over_ranks(dist, e0.elapsed_time(e1))
    if dist:
        dist.barrier()
    ms_step = ms / K
    value = NB * K / (ms * 1e-3)       # tokens of the sequences all ranks decode

    # e2e through the host-driven entry (host tokens/pos in, host tokens out)
    pos = P + W + K
    if NB > 1:
        t = np.zeros(NB, np.int32)
        B.check(L.dsv4b_model_decode_batch(model.h, np.zeros(NB, np.int32).ctypes.data, pos, t.ctypes.data),
                "dsv4b_model_decode_batch")
        pos += 1
        for _ in range(3):
            t = model.decode_batch(t, pos)
            pos += 1
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            t = model.decode_batch(t, pos)
            pos += 1
    else:
        tok = np.zeros(1, np.int32)
        B.check(L.dsv4_cuda_model_step(model.h, tok.ctypes.data, None), "dsv4_cuda_model_step")
        pos += 1
        t = int(tok[0])
        for _ in range(3):
            t = model.decode(t, pos)
            pos += 1
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            t = model.decode(t, pos)
            pos += 1
    e2e_s = (time.perf_counter() - t0) / n_e2e
    e2e_s = max_over_ranks(dist, e2e_s)

    peak, src = peaks()
    peak *= world                      # the ranks' HBM together
    bytes_tok = np.mean([decode_bytes_per_step(d, P + W + i, NB) for i in range(0, K, max(1, K // 16))])
    ach = bytes_tok / (ms_step * 1e-3) / 1e9
    out = {
        "metric": decode_metric(NB),
        "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp8 e4m3 / fp4 e2m1 / bf16 weights, f32 activations, f64 row sums",
        "data": "synthetic (random-init weights generated on device, random 512-token prompt)",
        "config": {"workload": "decode config 5 (Flash-scale synthetic)", "batch": NB,
                   "context": "%d-token prompt" % P, "positions": "%d..%d" % (P + W, P + W + K - 1),
                   "layers": d["n_layers"], "hidden": d["hidden"], "experts": d["n_experts"],
                   "topk": d["topk"], "vocab": d["vocab"],
                   "resident_gb": round(resident / 1e9, 1), "create_s": round(t_create, 1),
                   "l2": "no flush: each step streams %.1f GB of distinct weights (> 126 MB L2)"
                         % (bytes_tok / 1e9),
                   "parallelism": ("one sequence sharded over %d GPUs: expert inter slices, q heads / "
                                   "o_groups, wo_b columns, LM-head vocabulary; 2 sums per layer as "
                                   "one-shot exchanges over NVLink peer memory (%s) + 1 NCCL argmax "
                                   "all-gather per token"
                                   % (world, "NCCL all-reduce: DSV4B_PEER=0"
                                      if os.environ.get("DSV4B_PEER") == "0" else "CUDA IPC mailboxes")
                                   if world > 1 else
                                   "single GPU" + (", %d sequences stepped together (one GEMV item per "
                                                   "sequence, every other launch over all of them)" % NB
                                                   if NB > 1 else ""))},
        "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s",
                     "frac": ach / peak,
                     "peak_source": src + " burst hbm_gbs" + (" x %d GPUs" % world if world > 1 else ""),
                     "scope": ("whole decode token (one graph replay, %d kernels)" % launches_per_step
                               if NB == 1 else "whole batched step of %d tokens (one graph replay, %d kernels; "
                               "routed experts counted as the expected %.0f distinct per layer)"
                               % (NB, launches_per_step, expected_experts(d, NB))),
                     "bytes_per_unit": bytes_tok,
                     "traffic": (TRAFFIC_DECODE[0] + (bytes_tok - TRAFFIC_DECODE[1])
                                 if world == 1 and NB == 1 else None),
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum over one token's "
                                       "launches (profiles/decode_flash_c5_traffic.md), shifted to these "
                                       "positions by their algorithmic KV bytes" if world == 1 and NB == 1
                                       else "not captured for this step"},
        "gpu_launches": launches_per_step * K,
        "clocks": clk.summary(),
        "e2e": {"value": NB / e2e_s, "unit": "tok/s", "ms_per_step": e2e_s * 1e3,
                "h2d_bytes_per_step": 8 * NB, "d2h_bytes_per_step": 4 * NB,
                "api": ("dsv4_cuda_model_decode (host token, pos -> host next token), wall clock" if NB == 1 else
                        "dsv4b_model_decode_batch (host tokens, pos -> host next tokens), wall clock")},
    }
    if rank == 0 and world == 1 and not a.no_cpu:
        # the reference decodes one sequence at a time: its tok/s is the
        # batch-1 rate whatever the batch
        s_tok, _, desc, _ = cpu_decode_sample(8)
        out["cpu_baseline"] = {"value": 1.0 / s_tok, "unit": "tok/s",
                               "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count())),
                               "kind": "reference", "sample": desc}
    if world > 1 and L.dsv4b_model_comm_status(model.h) != 0:
        out["comm_error"] = "a peer exchange timed out waiting for a rank: results invalid"
    if rank == 0:
        print(json.dumps(out))
    model.close()
    L.dsv4_cuda_shutdown()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------- prefill

def cpu_prefill_sample(chunk, n_pass=2):
    """The reference's batched prompt path (dsv4_layer_forward_n in passes of
    chunk tokens, oracle/_ref) on the 3-layer Flash-geometry sample: a random
    prompt of n_pass passes, per-layer pass times scaled to the 43-layer mix.
    Returns (seconds per prompt token, description)."""
    import oracle as O
    import dsv4_model as M
    full = layer_ratios(M.flash_config())
    count = {r: full.count(r) for r in set(full)}
    d = M.flash_sample_config()
    t0 = time.perf_counter()
    sm = M.SyntheticModel(d, seed=0, fast=True)
    t_build = time.perf_counter() - t0
    n = chunk * n_pass
    prompt = np.random.default_rng(0).integers(0, d["vocab"], n).astype(np.int32)
    t0 = time.perf_counter()
    _, tp = O.model_prefill_ref(sm, prompt, 0, n + 1, chunk)
    t_run = time.perf_counter() - t0
    per_pass = tp[:, 0] * count[0] + tp[:, 1] * count[4] + tp[:, 2] * count[128]
    desc = ("reference dsv4_layer_forward_n in passes of %d (oracle/_ref, the --batch prompt path of "
            "src/cli/dsv4_run.c:391-442) on a 3-layer Flash-geometry sample (ratios 0/4/128, 256 experts), "
            "positions 0..%d, per-layer pass times scaled to the 43-layer mix (%d/%d/%d), the one LM head "
            "of the prompt left out; OMP_NUM_THREADS=%s; sample build %.0f s, run %.0f s"
            % (chunk, n - 1, count[0], count[4], count[128],
               os.environ.get("OMP_NUM_THREADS", "all %d" % os.cpu_count()), t_build, t_run))
    return float(np.sum(per_pass) / n), desc


def run_prefill(a):
    import torch
    import dsv4_b200 as B
    import dsv4_model as M
    if a.gpus != 1:
        raise SystemExit("prefill runs on one GPU (a one-sequence model)")
    L = B.init()
    d = M.flash_config()
    W, K, P, CH = max(a.warmup, 3), a.steps, a.context, a.chunk
    t0 = time.perf_counter()
    model = B.Model(M.ConfigOnly(d), P + 8, synthetic_seed=1234)
    t_create = time.perf_counter() - t0
    prompt = np.random.default_rng(0).integers(0, d["vocab"], P).astype(np.int32)
    stream = torch.cuda.ExternalStream(L.dsv4b_model_stream(model.h))
    # the prompt through per-token decode steps (the graph generate() runs),
    # for comparison
    model.begin(prompt)
    torch.cuda.synchronize()
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record(stream)
    for _ in range(P):
        B.check(L.dsv4b_model_step_async(model.h, None), "dsv4b_model_step_async")
    eb.record(stream)
    torch.cuda.synchronize()
    per_token_s = ea.elapsed_time(eb) * 1e-3
    # warm-up: each pass shape runs eagerly, then is captured, then replayed
    for _ in range(W):
        first = model.prefill(prompt, CH)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(torch.cuda.current_device()) as clk:
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(K):
            if model.prefill(prompt, CH) != first:
                raise SystemExit("prefill is not deterministic")
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    kernels = L.dsv4b_model_prefill_kernels(model.h)
    ms_step = ms / K
    value = P * K / (ms * 1e-3)
    # e2e: the C-ABI call on wall clock (host prompt in, first token out)
    t0 = time.perf_counter()
    for _ in range(K):
        model.prefill(prompt, CH)
    e2e_s = (time.perf_counter() - t0) / K
    peak, src = peaks()
    byts = prefill_bytes(d, P, CH)
    ach = byts / (ms_step * 1e-3) / 1e9
    n_pass = -(-P // CH)
    out = {
        "metric": prefill_metric(P, CH),
        "value": value, "unit": "tok/s", "n_gpus": 1, "steps": K, "warmup": W,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp8 e4m3 / fp4 e2m1 / bf16 weights, f32 activations, f64 row sums",
        "data": "synthetic (random-init weights generated on device, random %d-token prompt)" % P,
        "config": {"workload": "prefill config 5 (Flash-scale synthetic)", "prompt": P, "chunk": CH,
                   "passes": n_pass, "layers": d["n_layers"], "experts": d["n_experts"], "topk": d["topk"],
                   "vocab": d["vocab"], "create_s": round(t_create, 1),
                   "step": "one whole prefill (dsv4b_model_prefill: reset, %d passes, the head on the last "
                           "token), each pass a replayed graph" % n_pass,
                   "per_token_prompt_tok_s": P / per_token_s,
                   "l2": "no flush: each pass streams > 10 GB of distinct weights (> 126 MB L2)"},
        "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                     "peak_source": src + " burst hbm_gbs",
                     "scope": "whole prefill (every pass's launches)",
                     "bytes_per_unit": byts, "traffic": None,
                     "traffic_source": "not captured for this workload"},
        "gpu_launches": kernels * K if kernels > 0 else None,
        "clocks": clk.summary(),
        "e2e": {"value": P / e2e_s, "unit": "tok/s", "ms_per_step": e2e_s * 1e3,
                "h2d_bytes_per_step": 4 * P + 8 * P + 8, "d2h_bytes_per_step": 4,
                "api": "dsv4b_model_prefill (host prompt -> host first token), wall clock"},
    }
    if not a.no_cpu:
        s_tok, desc = cpu_prefill_sample(CH)
        out["cpu_baseline"] = {"value": 1.0 / s_tok, "unit": "tok/s",
                               "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count())),
                               "kind": "reference", "sample": desc}
    print(json.dumps(out))
    model.close()
    L.dsv4_cuda_shutdown()


# -------------------------------------------------------------- GEMV (C1)

def cpu_reference_gemv(seconds, threads=None):
    """The reference's CPU dsv4_matmul_fp8 on config 1, cycling weight copies
    larger than the LLC (reference bench/gemm_bw.c:11-26), best of the runs
    (bench/matmul_bw.c:96-99) over a bounded time budget."""
    import oracle as O
    import dsv4_quant as Q
    kind = "reference" if os.path.exists(O.REF_SO) else "port"
    chk = O.Checker(kind)
    W, S, x = Q.c1_gemv(seed=0)
    copies = [W] + [np.roll(W, i + 1, axis=0) for i in range(3)]   # 117 MB > LLC
    best, n, t_end = 1e9, 0, time.perf_counter() + seconds
    while time.perf_counter() < t_end or n < 3:
        t0 = time.perf_counter()
        chk.gemv_fp8(x, copies[n % len(copies)], S, C1_ROWS, C1_COLS)
        best = min(best, time.perf_counter() - t0)
        n += 1
    cores = threads or os.cpu_count()
    return {"value": C1_BYTES / best / 1e9, "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": "%d config-1 GEMVs over %d rotating weight copies (117 MB), best of runs, "
                      "OMP_NUM_THREADS=%s" % (n, len(copies), os.environ.get("OMP_NUM_THREADS", cores))}


def reference_gpu_gemv(W, S, x, ours_y, calls=400):
    """The reference's own GPU co-processor on config 1: its k_mmq_fp8 through
    its dsv4_cuda_mmq (src/cuda/dsv4_cuda.cu:93-129, 387-403), compiled
    unchanged for sm_100a into oracle/_ref/libdsv4ref_cuda.so. The call is
    host-to-host (pinned staging, two blocking copies, one launch), timed by
    the wall clock, the way its own bench/gpu_call.c times it; its output is
    checked against ours (vector-scaled relative error)."""
    import ctypes as C
    import oracle as O
    import dsv4_b200 as B
    path = os.path.join(os.path.dirname(O.REF_SO), "libdsv4ref_cuda.so")
    if not os.path.exists(path):
        return {"unavailable": "oracle/_ref/libdsv4ref_cuda.so not built"}
    L = C.CDLL(path)
    L.dsv4_cuda_init.restype = C.c_int
    L.dsv4_cuda_upload.restype = C.c_int
    if L.dsv4_cuda_init() != 0:
        return {"unavailable": "reference dsv4_cuda_init failed"}
    Wc, Sc = np.ascontiguousarray(W), np.ascontiguousarray(S)
    q = B.QMat(Wc.ctypes.data, Sc.ctypes.data, B.WFP8, C1_ROWS, C1_COLS, 128, 128)
    if L.dsv4_cuda_upload(C.byref(q)) != 0:
        return {"unavailable": "reference dsv4_cuda_upload failed"}
    y = np.empty(C1_ROWS, np.float32)
    for _ in range(5):
        L.dsv4_cuda_mmq(y.ctypes.data, x.ctypes.data, C.byref(q))
    ts = []
    for _ in range(calls):
        t0 = time.perf_counter()
        L.dsv4_cuda_mmq(y.ctypes.data, x.ctypes.data, C.byref(q))
        ts.append(time.perf_counter() - t0)
    L.dsv4_cuda_shutdown()
    ref = np.asarray(ours_y, np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    vrel = float(np.max(np.abs(y - ref) / np.maximum(rms, np.maximum(np.abs(y), np.abs(ref)))))
    best, med = min(ts), float(np.median(ts))
    return {"kernel": "k_mmq_fp8 (reference src/cuda/dsv4_cuda.cu, unchanged, sm_100a)",
            "call_ms_median": med * 1e3, "call_ms_best": best * 1e3,
            "call_gbs_median": C1_BYTES / med / 1e9, "call_gbs_best": C1_BYTES / best / 1e9,
            "timing": "wall clock per dsv4_cuda_mmq (host x -> host y), %d calls" % calls,
            "vrel_vs_ours": vrel}


def run_gemv(a):
    import torch
    import dsv4_b200 as B
    import dsv4_quant as Q
    rank, world, dist = dist_setup(a.gpus)
    L = B.init()
    W, S, x = Q.c1_gemv(seed=0)
    mats = []
    for i in range(NCOPY):                       # distinct bytes per copy
        Wi = W if i == 0 else np.roll(W, i, axis=1)
        m = B.Matrix(B.WFP8, Wi, S)
        B.check(m.upload(), "upload")
        mats.append(m)
    dev = torch.cuda.current_device()
    stream = torch.cuda.Stream()
    tx = torch.from_numpy(x).cuda()
    ty = torch.empty(C1_ROWS, dtype=torch.float32, device="cuda")
    ptrs = [m.device_ptrs() for m in mats]

    def step(i):
        dw, ds = ptrs[i % NCOPY]
        B.gemv(B.WFP8, ty, tx, dw, ds, C1_ROWS, C1_COLS, 128, 128, 1, stream)

    # Launch cost is not the kernel's: the K timed steps replay CUDA graphs of
    # up to 1000 captured GEMVs each (weights rotating over the 8 copies).
    with torch.cuda.stream(stream):
        for i in range(max(a.warmup, 3)):
            step(i)
    torch.cuda.synchronize()
    chunk = min(a.steps, 1000)
    plan = [(chunk, a.steps // chunk)] + ([(a.steps % chunk, 1)] if a.steps % chunk else [])
    graphs = []
    for n, reps in plan:
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            for i in range(n):
                step(i)
        graphs.append((gr, reps))
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev) as clk:
        t_end = time.perf_counter() + 0.5          # load the GPU while sampling starts
        while time.perf_counter() < t_end:
            with torch.cuda.stream(stream):
                graphs[0][0].replay()
            torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            e0.record(stream)
            for gr, reps in graphs:
                for _ in range(reps):
                    gr.replay()
            e1.record(stream)
        torch.cuda.synchronize()
    ms = max_over_ranks(dist, e0.elapsed_time(e1))
    ms_step = ms / a.steps
    value = world * C1_BYTES / (ms_step * 1e-3) / 1e9

    # e2e: the reference-facing call, host buffers, copies inside the region
    for i in range(3):
        mats[i % NCOPY].mmq(x)
    ke = max(50, min(a.steps // 4, 2000))
    t0 = time.perf_counter()
    for i in range(ke):
        mats[i % NCOPY].mmq(x)
    e2e_s = max_over_ranks(dist, (time.perf_counter() - t0) / ke)
    e2e = {"value": world * C1_BYTES / e2e_s / 1e9, "unit": "GB/s", "ms_per_step": e2e_s * 1e3,
           "h2d_bytes_per_step": C1_COLS * 4, "d2h_bytes_per_step": C1_ROWS * 4,
           "api": "dsv4_cuda_mmq (host x -> host y), wall clock"}

    peak, src = peaks()
    ach = C1_BYTES / (ms_step * 1e-3) / 1e9
    out = {
        "metric": GEMV_METRIC,
        "value": value, "unit": "GB/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "e4m3 weights, f32 x, f64 accumulation", "data": "synthetic",
        "config": {"workload": "gemv_fp8 config 1", "rows": C1_ROWS, "cols": C1_COLS, "batch": 1,
                   "l2": "8 rotating resident weight copies (235 MB > 126 MB L2)",
                   "parallelism": "replica per GPU" if world > 1 else "single GPU"},
        "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s",
                     "frac": ach / peak,
                     "peak_source": src + " burst hbm_gbs" + (" x %d GPUs" % world if world > 1 else ""),
                     "scope": "k_gemv_group, one launch per step", "bytes_per_unit": C1_BYTES,
                     "traffic": TRAFFIC_C1},
        "gpu_launches": a.steps,
        "clocks": clk.summary(),
        "e2e": e2e,
    }
    if rank == 0 and world == 1 and not a.no_cpu:
        out["cpu_baseline"] = cpu_reference_gemv(10.0)
    if rank == 0 and world == 1:
        # the same call of ours, host to host, beside the reference GPU kernel's
        y0 = mats[0].mmq(x)
        out["reference_gpu"] = reference_gpu_gemv(W, S, x, y0)
        out["reference_gpu"]["ours_e2e_gbs"] = e2e["value"]
    if rank == 0:
        print(json.dumps(out))
    L.dsv4_cuda_shutdown()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------- MoE (C2)

MOE_METRIC = "routed MoE FFN token HBM GB/s (config 2: 256 FP4 experts top-6 + shared FP8, fp32 sigmoid router)"
C2_H, C2_I, C2_E, C2_K = 4096, 2048, 256, 6
# one token: 6 routed experts (w1, w3 2048x4096, w2 4096x2048 in e2m1 + 1x32
# E8M0) + the shared FP8 expert + the fp32 router + x and the output
C2_BYTES = 6 * 13369344 + 25167360 + 4194304 + 32768


def build_moe(seed=0):
    """Config 2's layer: experts N(0, 0.02) quantised to e2m1 with ue8m0 1x32
    scales on the GPU (bit-identical to dsv4_quant.quant_fp4), shared expert
    FP8 128x128, fp32 router N(0, 0.02). Returns host matrices (resident)."""
    import torch
    import dsv4_b200 as B
    import dsv4_quant as Q
    tg = torch.Generator(device="cuda").manual_seed(seed)
    experts = []
    for e in range(C2_E):
        trio = []
        for rows, cols in ((C2_I, C2_H), (C2_I, C2_H), (C2_H, C2_I)):
            Wt, St = Q.quant_fp4_torch(torch.randn((rows, cols), generator=tg, device="cuda") * 0.02)
            m = B.Matrix(B.WFP4, Wt.cpu().numpy(), St.cpu().numpy())
            B.check(m.upload(), "upload")
            trio.append(m)
        experts.append(trio)
    rng = np.random.default_rng(seed)
    shared = []
    for rows, cols in ((C2_I, C2_H), (C2_I, C2_H), (C2_H, C2_I)):
        W, S = Q.quant_fp8(rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02), 128)
        m = B.Matrix(B.WFP8, W, S)
        B.check(m.upload(), "upload")
        shared.append(m)
    gate = B.Matrix(B.WF32, (rng.standard_normal((C2_E, C2_H)) * 0.02).astype(np.float32))
    B.check(gate.upload(), "upload")
    torch.cuda.synchronize()
    return gate, experts, shared


def cpu_moe_token(ref, port, x, gate, experts, shared):
    """One config-2 token on the host: the reference's own kernels for the
    experts (dsv4_matmul_fp4, dsv4_swiglu, dsv4_matmul_fp8), the restated
    fp32 router and sigmoid top-6 (the reference C has neither), the k-ordered
    combine of src/model/dsv4_layer.c:471-483."""
    logits = port.gemv_f32(x, gate.W, C2_E, C2_H)
    idx, w = port.route(logits, C2_K, 1.0, score_func=2)
    out = np.zeros(C2_H, np.float32)
    for k in range(C2_K):
        w1, w3, w2 = experts[idx[k]]
        g = ref.gemv_fp4(x, w1.W, w1.S, C2_I, C2_H)
        u = ref.gemv_fp4(x, w3.W, w3.S, C2_I, C2_H)
        h = ref.swiglu(g, u, 10.0)
        acc = ref.gemv_fp4(h, w2.W, w2.S, C2_H, C2_I)
        out = out + np.float32(w[k]) * acc
    g = ref.gemv_fp8(x, shared[0].W, shared[0].S, C2_I, C2_H)
    u = ref.gemv_fp8(x, shared[1].W, shared[1].S, C2_I, C2_H)
    return out + ref.gemv_fp8(ref.swiglu(g, u, 10.0), shared[2].W, shared[2].S, C2_H, C2_I)


def cpu_moe_sample(gate, experts, shared, seconds):
    import oracle as O
    kind = "reference" if os.path.exists(O.REF_SO) else "port"
    ref, port = O.Checker(kind), O.Checker("port")
    rng = np.random.default_rng(7)
    n, t_end, t0 = 0, time.perf_counter() + seconds, time.perf_counter()
    while time.perf_counter() < t_end or n < 2:
        cpu_moe_token(ref, port, rng.standard_normal(C2_H, dtype=np.float32), gate, experts, shared)
        n += 1
    per = (time.perf_counter() - t0) / n
    return per, n, kind


def run_moe(a):
    import torch
    import dsv4_b200 as B
    rank, world, dist = dist_setup(a.gpus)
    L = B.init()
    t0 = time.perf_counter()
    gate, experts, shared = build_moe()
    t_build = time.perf_counter() - t0
    moe = B.MoE(gate, experts, shared, topk=C2_K, route_scale=1.0, score_func=2, swiglu_limit=10.0)
    st = torch.cuda.Stream()
    W, K = max(a.warmup, 3), a.steps
    xs = torch.randn((W + K, C2_H), device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
    out = torch.empty(C2_H, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")     # > 126 MB L2
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    with torch.cuda.stream(st):
        for i in range(W):
            moe.forward_dev(out, xs[i], st)
    torch.cuda.synchronize()
    with Clocks(torch.cuda.current_device()) as clk:
        with torch.cuda.stream(st):
            for i in range(K):
                flush.zero_()
                ev[i][0].record(st)
                moe.forward_dev(out, xs[W + i], st)
                ev[i][1].record(st)
        torch.cuda.synchronize()
    ms = max_over_ranks(dist, sum(e0.elapsed_time(e1) for e0, e1 in ev))
    ms_step = ms / K
    value = C2_BYTES / (ms_step * 1e-3) / 1e9
    # e2e: the host-buffer call dsv4_cuda_moe (host x in, host output out)
    xh = np.random.default_rng(3).standard_normal((64, C2_H), dtype=np.float32)
    for i in range(3):
        moe(xh[i])
    t0 = time.perf_counter()
    for i in range(64):
        moe(xh[i])
    e2e_s = (time.perf_counter() - t0) / 64
    peak, src = peaks()
    out_line = {
        "metric": MOE_METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms_step, "tokens_per_s": 1e3 / ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e2m1 / e4m3 / f32 weights, f32 activations, f64 row sums",
        "data": "synthetic (config 2 distributions, quantised on the GPU)",
        "config": {"workload": "moe config 2 (one token)", "hidden": C2_H, "experts": C2_E, "inter": C2_I,
                   "topk": C2_K, "router": "fp32 sigmoid", "build_s": round(t_build, 1),
                   "l2": "flushed (256 MB write) before every timed step; a distinct x (routing) per step"},
        "roofline": {"bound": "hbm", "achieved": value, "peak": peak, "unit": "GB/s", "frac": value / peak,
                     "peak_source": src + " burst hbm_gbs", "scope": "one token: router + 6 experts + shared "
                     "(%d launches, CUDA events around each token)" % 4, "bytes_per_unit": C2_BYTES,
                     "traffic": None},
        "gpu_launches": 4 * K,
        "clocks": clk.summary(),
        "e2e": {"value": C2_BYTES / e2e_s / 1e9, "unit": "GB/s", "ms_per_step": e2e_s * 1e3,
                "h2d_bytes_per_step": C2_H * 4, "d2h_bytes_per_step": C2_H * 4 + C2_K * 8,
                "api": "dsv4_cuda_moe (host x -> host output, selection, weights), wall clock"},
    }
    if rank == 0 and world == 1 and not a.no_cpu:
        per, n, kind = cpu_moe_sample(gate, experts, shared, 10.0)
        out_line["cpu_baseline"] = {"value": C2_BYTES / per / 1e9, "unit": "GB/s",
                                    "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count())),
                                    "kind": kind, "sample": "%d config-2 tokens (reference dsv4_matmul_fp4 / "
                                    "dsv4_swiglu / dsv4_matmul_fp8, restated fp32 sigmoid router), %.1f ms each"
                                    % (n, per * 1e3)}
    if rank == 0:
        print(json.dumps(out_line))
    moe.close()
    L.dsv4_cuda_shutdown()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------- sparse MLA (C3)

MLA_METRIC = "sparse-MLA decode step HBM GB/s (config 3: 32768 positions, indexer 64x128 e4m3, top-2048, 64 heads x 576)"
C3_N, C3_H, C3_D, C3_HI, C3_DI, C3_K = 32768, 64, 576, 64, 128, 2048
# per sequence: e4m3 keys + the selected bf16 KV rows + q (f32, attention and
# indexer) + head weights + the score vector written and read + the output
C3_BYTES = C3_N * C3_DI + C3_K * C3_D * 2 + (C3_H * C3_D + C3_HI * C3_DI + C3_HI) * 4 + 2 * C3_N * 4 + \
    C3_K * 4 + C3_H * C3_D * 4
C3_FLOPS = 2 * (C3_N * C3_HI * C3_DI + 2 * C3_K * C3_H * C3_D)


def run_mla(a):
    import torch
    import dsv4_b200 as B
    rank, world, dist = dist_setup(a.gpus)
    B.init()
    bt = a.batch
    nset = max(1, -(-4 // bt))                   # >= 4 distinct sequences: > 126 MB L2 every step
    g = torch.Generator(device="cuda").manual_seed(0)
    sets = []
    for _ in range(nset):
        kv = torch.randn((bt, C3_N, C3_D), generator=g, device="cuda").to(torch.bfloat16)
        keys = torch.randn((bt, C3_N, C3_DI), generator=g, device="cuda").to(torch.float8_e4m3fn)
        q = torch.randn((bt, C3_H, C3_D), generator=g, device="cuda")
        qi = torch.randn((bt, C3_HI, C3_DI), generator=g, device="cuda")
        w = torch.randn((bt, C3_HI), generator=g, device="cuda")
        sets.append((kv, keys, q, qi, w))
    sink = torch.randn(C3_H, generator=g, device="cuda")
    scores = torch.empty((bt, C3_N), device="cuda")
    idx = torch.empty((bt, C3_K), dtype=torch.int32, device="cuda")
    o = torch.empty((bt, C3_H, C3_D), device="cuda")
    scratch = torch.empty(B.sparse_attn_scratch(C3_H, C3_D, C3_K, bt), dtype=torch.uint8, device="cuda")
    iscale = float(np.float32(1 / np.sqrt(np.float32(C3_DI))) * np.float32(1 / np.sqrt(np.float32(C3_HI))))
    scale = float(np.float32(1.0) / np.sqrt(np.float32(C3_D)))
    st = torch.cuda.Stream()

    def step(i):
        kv, keys, q, qi, w = sets[i % nset]
        B.indexer_score_dev(scores, qi, keys.view(torch.uint8), B.E4M3, C3_DI, C3_N * C3_DI, w, C3_HI, C3_DI,
                            C3_N, iscale, bt, st)
        B.topk_dev(idx, scores, C3_N, C3_K, bt, st)
        B.sparse_attn_dev(o, q, kv.view(torch.int16), B.BF16, C3_N, sink, idx, C3_H, C3_D, C3_K, scale, bt,
                          scratch, st)

    W, K = max(a.warmup, 3), a.steps
    with torch.cuda.stream(st):
        for i in range(W):
            step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(torch.cuda.current_device()) as clk:
        with torch.cuda.stream(st):
            e0.record(st)
            for i in range(K):
                step(i)
            e1.record(st)
        torch.cuda.synchronize()
    ms = max_over_ranks(dist, e0.elapsed_time(e1))
    ms_step = ms / K
    value = bt * C3_BYTES / (ms_step * 1e-3) / 1e9
    # e2e: the reference-signature host calls, one sequence at a time (host
    # keys widened to f32 and host KV as the reference's dsv4_indexer_score /
    # dsv4_topk / dsv4_sparse_attn take them)
    kv, keys, q, qi, w = sets[0]
    kvh = kv[0].float().cpu().numpy()
    kh = keys[0].float().cpu().numpy()
    qh, qih, wh, sh = q[0].cpu().numpy(), qi[0].cpu().numpy(), w[0].cpu().numpy(), sink.cpu().numpy()
    ne = 3
    t0 = time.perf_counter()
    for _ in range(ne):
        sc = B.indexer_score(qih, kh, wh)
        ii = B.topk(sc, C3_K)
        B.sparse_attn(qh, kvh, sh, ii, scale)
    e2e_s = (time.perf_counter() - t0) / ne
    h2d = C3_HI * C3_DI * 4 + C3_N * C3_DI * 4 + C3_HI * 4 + C3_N * 4 + C3_H * C3_D * 4 + C3_N * C3_D * 4 + \
        C3_H * 4 + C3_K * 4
    d2h = C3_N * 4 + C3_K * 4 + C3_H * C3_D * 4
    peak, src = peaks()
    tc = 1622.1
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            tc = float(json.load(f)["bf16_tflops"])
    except Exception:
        pass
    flops_s = bt * C3_FLOPS / (ms_step * 1e-3)
    out_line = {
        "metric": MLA_METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms_step, "sequences_per_s": bt / (ms_step * 1e-3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 keys / bf16 KV, f64 indexer dots, f32 attention",
        "data": "synthetic (config 3 distributions)",
        "config": {"workload": "mla config 3", "batch": bt, "positions": C3_N, "heads": C3_H, "d": C3_D,
                   "index_heads": C3_HI, "index_dim": C3_DI, "topk": C3_K,
                   "l2": "%d distinct sequence sets rotated (%.0f MB of keys + KV per step set)"
                         % (nset, bt * (C3_N * C3_D * 2 + C3_N * C3_DI) / 1e6)},
        "roofline": {"bound": "hbm", "achieved": value, "peak": peak, "unit": "GB/s", "frac": value / peak,
                     "peak_source": src + " burst hbm_gbs", "bytes_per_unit": C3_BYTES,
                     "scope": "indexer + top-k + attention per step (4 launches)",
                     "flops_per_unit": C3_FLOPS, "achieved_tflops": flops_s / 1e12,
                     "tensor_peak_tflops": tc, "tensor_frac": flops_s / 1e12 / tc,
                     "note": "the indexer's dots run in exact f64 (bit-identical scores); that, not HBM, bounds it",
                     "traffic": None},
        "gpu_launches": 4 * K,
        "clocks": clk.summary(),
        "e2e": {"value": C3_BYTES / e2e_s / 1e9, "unit": "GB/s", "ms_per_step": e2e_s * 1e3,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "dsv4_cuda_indexer_score / topk / sparse_attn, one sequence, host buffers"},
    }
    if rank == 0 and world == 1 and not a.no_cpu:
        out_line["cpu_baseline"] = cpu_mla_sample(qih, kh, wh, qh, kvh, sh, scale)
    if rank == 0:
        print(json.dumps(out_line))
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def cpu_mla_sample(qi, keys, w, q, kv, sink, scale, k_small=256):
    """One config-3 sequence through the reference's own C (oracle/_ref):
    dsv4_indexer_score at full size, dsv4_topk at k = 256 (its repeated
    argmax is O(n k); the time is scaled by 2048 / 256 to the config's k),
    dsv4_sparse_attn over the 2048 selected rows."""
    import oracle as O
    kind = "reference" if os.path.exists(O.REF_SO) else "port"
    ref = O.Checker(kind)
    t0 = time.perf_counter()
    sc = ref.indexer_score(qi, keys, w, C3_HI, C3_DI)
    t1 = time.perf_counter()
    ref.topk(sc, k_small)
    t2 = time.perf_counter()
    ii = O.Checker("port").topk(sc, C3_K)
    t3 = time.perf_counter()
    ref.sparse_attn(q, kv, sink, ii, scale)
    t4 = time.perf_counter()
    per = (t1 - t0) + (t2 - t1) * (C3_K / k_small) + (t4 - t3)
    return {"value": C3_BYTES / per / 1e9, "unit": "GB/s",
            "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count())), "kind": kind,
            "sample": "one sequence: indexer %.0f ms, top-%d %.0f ms scaled x%d, attention %.0f ms"
                      % ((t1 - t0) * 1e3, k_small, (t2 - t1) * 1e3, C3_K // k_small, (t4 - t3) * 1e3)}


# ------------------------------------------------------- reference arm

def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if a.workload == "prefill":
        s_tok, desc = cpu_prefill_sample(a.chunk)
        v = 1.0 / s_tok
        print(json.dumps({
            "metric": prefill_metric(a.context, a.chunk), "value": v, "unit": "tok/s", "impl": "reference",
            "n_gpus": a.gpus, "steps": 1, "warmup": 0, "ms_per_step": s_tok * a.context * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp8 e4m3 / fp4 e2m1 / bf16 weights, f32 activations, f64 row sums",
            "data": "synthetic (random-init weights, random prompt)",
            "config": {"workload": "prefill config 5 (Flash-scale synthetic)", "prompt": a.context,
                       "chunk": a.chunk, "layers": "43 (3 timed, per-layer times scaled to the 43-layer mix)",
                       "sample": "the first 2 passes of the prompt"},
            "cpu_baseline": {"value": v, "unit": "tok/s",
                             "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count())),
                             "kind": "reference", "sample": desc},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return
    if a.workload == "decode":
        # the GPU arm's first positions after the same prompt and warm-up (a
        # bounded sample of them: minutes, not hours)
        n = max(4, min(a.steps, 32))
        W = max(a.warmup, 3)
        s_tok, per, desc, first = cpu_decode_sample(n, warm=W, prompt_len=a.context)
        v = 1.0 / s_tok
        print(json.dumps({
            "metric": decode_metric(a.batch), "value": v, "unit": "tok/s", "impl": "reference",
            "n_gpus": a.gpus, "steps": n, "warmup": W, "ms_per_step": s_tok * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp8 e4m3 / fp4 e2m1 / bf16 weights, f32 activations, f64 row sums",
            "data": "synthetic (random-init weights, the GPU arm's random %d-token prompt)" % a.context,
            "config": {"workload": "decode config 5 (Flash-scale synthetic)", "batch": a.batch,
                       "context": "%d-token prompt" % a.context,
                       "positions": "%d..%d" % (first, first + n - 1),
                       "layers": "43 (3 timed, per-layer times scaled to the 43-layer mix)",
                       "batching": ("the reference decodes one sequence at a time (its batched layer, "
                                    "dsv4_layer_forward_n, takes tokens of one sequence): %d sequences take "
                                    "%d times one, so its tok/s is the batch-1 rate" % (a.batch, a.batch)
                                    if a.batch > 1 else "one sequence")},
            "cpu_baseline": {"value": v, "unit": "tok/s",
                             "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count())),
                             "kind": "reference", "sample": desc},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return
    secs = max(2.0, 20.0 / max(a.steps, 1))
    vals = []
    for _ in range(min(a.warmup, 3)):
        cpu_reference_gemv(0.5)
    base = None
    for _ in range(min(a.steps, 20)):
        base = cpu_reference_gemv(secs)
        vals.append(base["value"])
    v = float(np.median(vals))
    base["value"] = v
    print(json.dumps({
        "metric": GEMV_METRIC,
        "value": v, "unit": "GB/s", "impl": "reference", "n_gpus": a.gpus, "steps": a.steps,
        "warmup": a.warmup, "higher_is_better": True, "dtype": "e4m3 weights, f32 x, f64 accumulation",
        "data": "synthetic", "config": {"workload": "gemv_fp8 config 1", "rows": C1_ROWS, "cols": C1_COLS},
        "cpu_baseline": base,
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default 256 decode tokens / 20000 GEMVs)")
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "gemv_fp8", "moe", "mla"])
    ap.add_argument("--batch", type=int, default=1,
                    help="decode: sequences stepped together (config 5: 1 or 32); mla: sequences per step "
                         "(config 3: 1 or 8)")
    ap.add_argument("--context", type=int, default=512,
                    help="decode: prompt tokens before timing; prefill: the prompt's tokens")
    ap.add_argument("--chunk", type=int, default=32, help="prefill: tokens per pass (1..64)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    a = ap.parse_args()
    if a.steps is None:
        a.steps = {"decode": 256, "prefill": 3, "gemv_fp8": 20000, "moe": 200, "mla": 50}[a.workload]
    if a.impl == "reference":
        run_reference(a)
    elif a.workload == "decode":
        run_decode(a)
    elif a.workload == "prefill":
        run_prefill(a)
    elif a.workload == "moe":
        run_moe(a)
    elif a.workload == "mla":
        run_mla(a)
    else:
        run_gemv(a)


if __name__ == "__main__":
    main()
