"""Benchmark of the masked-selection path on B200.

Default workload (the batched verification round, 256 sequences x (K+1) = 9
rows of bfloat16 logits at V = 248,320 per GPU): one step is one verification
round -- the fused masked argmax + popcount kernel over all 2,304 rows plus the
acceptance/budget epilogue -- on inputs already resident in HBM.  Other
workloads: ``argmax`` (6 rows fp32, the reference's CPU-runnable case),
``sample`` (8 rows fp16 at T = 0.7, rotated through enough batches to exceed
L2) and ``scale`` (row-sharded bf16 rows).

Printed JSON keys beyond the driver contract: ``roofline`` (dominant kernel's
algorithmic bytes / its CUDA-event duration vs the measured HBM copy peak),
``cpu_baseline`` (the CPU oracle on this host's cores), ``clocks`` (nvidia-smi
samples during the measurement), ``gpu_launches`` and ``e2e`` (same metric
through the public API: masks, drafts and lengths copied host->device from
pinned memory and results read back every step; logits stay device-resident
as the model's output, exactly as the reference's select_token receives them).

``--impl reference`` times the reference algorithm's CPU restatement (the
oracle, all host threads) on the same workload instead.
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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "bitmask-speculation_b200"))
sys.path.insert(0, str(ROOT))

L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
# dram__bytes_read.sum + dram__bytes_write.sum per row from one ncu capture of the dominant kernel
# on a smaller case of the same workload; traffic grows with the rows processed.
NCU_TRAFFIC_PER_ROW = {"verify": 533530, "sample": 533980}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["verify", "grammar", "argmax", "sample", "scale", "vocab", "decode",
                                           "stochastic"],
                    default="verify")
    ap.add_argument("--prompts", type=int, default=32, help="prompts for the decode workload")
    ap.add_argument("--new-tokens", type=int, default=256, help="tokens generated per prompt (decode workload)")
    ap.add_argument("--seqs", type=int, default=256, help="verification sequences per GPU")
    ap.add_argument("--draft-noise", type=float, default=0.7,
                    help="stochastic workload: std of the noise between target and draft logits")
    ap.add_argument("--rows", type=int, default=8192, help="rows per GPU for the scale workload")
    ap.add_argument("--sample-rows", type=int, default=8,
                    help="rows per sampling batch (the 8 configuration rows tiled, fresh uniforms)")
    ap.add_argument("--sample-density", type=float, default=None,
                    help="override every sampling row's mask density (default: the configuration's mix)")
    ap.add_argument("--sample-dtype", choices=["float16", "bfloat16"], default="float16",
                    help="logits type of the sampling workload (the configuration's rows are fp16)")
    ap.add_argument("--p2p", action="store_true",
                    help="vocab workload: exchange the shard partials through peer memory instead of NCCL")
    ap.add_argument("--no-workspace", action="store_true",
                    help="run the selection kernels on their fixed schedule (no dynamic-schedule workspace)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-sampler-roofline", action="store_true",
                    help="skip the sampler's roofline lines (256 and 2,304 fp16 rows) of the default run")
    ap.add_argument("--roofline-seconds", type=float, default=1.5)
    ap.add_argument("--cluster", type=int, default=0,
                    help="force the selection kernel's cluster size (1/2/4/8/16; 0 = automatic)")
    ap.add_argument("--clusters", type=int, default=0,
                    help="force the number of persistent clusters (0 = automatic)")
    return ap.parse_args()


# ---------------------------------------------------------------- environment
def host_threads() -> int:
    """Host threads this process may run on (torchrun sets OMP_NUM_THREADS=1 for its ranks; the
    CPU arms ask for every core of the affinity mask explicitly)."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return max(1, os.cpu_count() or 1)


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self):
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [s for s, p in zip(sm, power) if p >= statistics.median(power)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power)}


# ---------------------------------------------------------------- workloads
class Workload:
    """Inputs and one step of the hot path on this rank's GPU."""

    def __init__(self, args, rank, device):
        import torch
        from bitmask_speculation_b200 import workloads as wl
        self.args = args
        self.device = device
        self.kind = args.workload
        vocab = wl.VOCAB
        self.vocab = vocab
        self.words = wl.words_for(vocab)
        if self.kind == "grammar":
            if args.impl == "reference":  # input synthesis on the host for the CPU arm
                import numpy as np
                import oracle

                def select(rows, masks):
                    bits = rows.cpu().view(torch.int16).numpy().view(np.uint16)
                    tok, _, st = oracle.reduce_rows(bits, masks, dtype="bfloat16", threads=host_threads())
                    return tok, st
            else:
                def select(rows, masks):
                    tok, _, st = self.native.masked_reduce_batch(rows, torch.from_numpy(masks).to(device))
                    return tok.cpu().numpy(), st.cpu().numpy()
            (self.logits, self.masks, self.proposals, self.lengths, self.grammars,
             self.drafts) = wl.grammar_round_torch(args.seqs, select, seed=11 + 1000 * rank, device=device)
            self.rows = self.logits.shape[0]
            self.batches = 1
            self.esize = 2
            self.dtype = "bf16"
            from bitmask_speculation_b200.scheduling import DensityPolicy
            self.policy = DensityPolicy().native()
            self.name = (f"grammar: {args.seqs} sequences x (K+1)=9 rows bf16 N(0,3^2) at V={vocab}, each under a "
                         "64-state token DFA (enum 1-8 / Bernoulli 0.3 states, EOS); drafts take the target's "
                         "masked choice with p=0.88; fork masks of the drafts")
        elif self.kind == "verify":
            self.logits, self.masks, self.proposals, self.lengths = wl.verify_batch_torch(
                args.seqs, seed=3 + 1000 * rank, device=device)
            self.rows = self.logits.shape[0]
            self.batches = 1
            self.esize = 2
            self.dtype = "bf16"
            from bitmask_speculation_b200.scheduling import DensityPolicy
            self.policy = DensityPolicy().native()
            self.name = (f"verify: {args.seqs} sequences x (K+1)=9 rows bf16 N(0,3^2) at V={vocab}; masks 40% "
                         "enum 2-32 / 30% Bernoulli 0.05 / 30% Bernoulli 0.6; drafts geometric (0.88)")
        elif self.kind == "argmax":
            values, masks = wl.argmax_config_np(seed=1 + rank)
            import numpy as np
            reps = max(1, int(2 * L2_BYTES // values.nbytes) + 1)  # rotate > L2 of distinct batches
            self.logits_all = torch.from_numpy(np.ascontiguousarray(np.tile(values, (reps, 1)))).to(device)
            self.masks_all = torch.from_numpy(np.ascontiguousarray(np.tile(masks, (reps, 1)))).to(device)
            self.rows = 6
            self.batches = reps
            self.esize = 4
            self.dtype = "f32"
            self.name = "argmax: 6 rows fp32 N(0,3^2) at V=248320 (masks .5/.5/4 valid/16 valid/.02/1 valid)"
        elif self.kind == "sample":
            import numpy as np
            densities = wl.SAMPLE_DENSITIES if args.sample_density is None else (args.sample_density,) * 8
            bits, masks, uniforms, temp = wl.sample_config_np(seed=2 + rank, densities=densities)
            tile = max(1, -(-args.sample_rows // bits.shape[0]))
            bits, masks = np.tile(bits, (tile, 1))[:args.sample_rows], np.tile(masks, (tile, 1))[:args.sample_rows]
            uniforms = np.random.default_rng(2 + rank).random(bits.shape[0])
            reps = max(1, int(2 * L2_BYTES // bits.nbytes) + 1)
            self.logits_all = torch.from_numpy(np.tile(bits, (reps, 1)).view(np.int16)).view(torch.float16).to(device)
            if args.sample_dtype == "bfloat16":
                self.logits_all = self.logits_all.to(torch.bfloat16)
            self.masks_all = torch.from_numpy(np.ascontiguousarray(np.tile(masks, (reps, 1)))).to(device)
            self.uniforms_all = torch.from_numpy(np.tile(uniforms, reps)).to(device)
            self.temperature = temp
            self.rows = bits.shape[0]
            self.batches = reps
            self.esize = 2
            self.dtype = "f16" if args.sample_dtype == "float16" else "bf16"
            self.name = (f"sample: {self.rows} rows {self.dtype} N(0,2^2) at V=248320, T=0.7, densities "
                         "{1,.5,.1,.01,1e-4,.9,.3,.05}")
        elif self.kind == "vocab":
            # Every rank builds the same full rows, keeps its vocabulary slice and the full masks.
            from bitmask_speculation_b200.sharding import shard_bounds
            import torch.distributed as dist
            world = dist.get_world_size() if dist.is_initialized() else 1
            full, self.masks = wl.scale_rows_torch(args.rows, seed=5, device=device)
            off, size = shard_bounds(vocab, world)[rank]
            self.logits = full[:, off:off + size].contiguous()
            del full
            self.world = world
            self.rows = args.rows
            self.batches = 1
            self.esize = 2
            self.dtype = "bf16"
            self.exchange = None
            if args.p2p:
                # Partials stored into every rank's exchange area by the selection kernel itself.
                from bitmask_speculation_b200.sharding import PeerExchange
                if world > 1:
                    self.exchange = PeerExchange(args.rows, device=device)
                else:
                    own, _ = PeerExchange.create(device, 1, args.rows)
                    self.exchange = PeerExchange(args.rows, areas=[own], rank=0, device=device)
            self.transport = ("peer-memory exchange of 32-byte partials (stores over NVLink from the selection "
                              "kernel, epoch flags)" if args.p2p else "NCCL all-gather of 32-byte partials")
            self.name = (f"vocab-sharded: {args.rows} rows bf16 N(0,3^2) at V=248320 split {world} ways, "
                         f"log-uniform mask density; {self.transport}")
        else:
            self.logits, self.masks = wl.scale_rows_torch(args.rows, seed=5 + 1000 * rank, device=device)
            self.rows = args.rows
            self.batches = 1
            self.esize = 2
            self.dtype = "bf16"
            self.name = f"scale: {args.rows} rows/GPU bf16 N(0,3^2) at V=248320, log-uniform mask density"
        self.step_index = 0
        self._alloc_outputs()

    @property
    def native(self):
        """The library's tensor front end (the b200 arm only: the reference arm never loads it)."""
        from bitmask_speculation_b200.kernels._extension import load_extension
        return load_extension()

    @property
    def bytes_per_row(self):
        if self.kind == "vocab":  # this rank's slice of the logits and of the mask words
            return self.logits.shape[1] * self.esize + (self.logits.shape[1] // 32) * 4 + 20
        return self.vocab * self.esize + self.words * 4 + 20

    @property
    def dtype_code(self):
        return {"f32": 0, "bf16": 1, "f16": 2}[self.dtype]

    def workspace(self):
        """(pointer, bytes) of the dynamic-schedule workspace, or (None, 0) with --no-workspace."""
        if self.args.no_workspace:
            return None, 0
        if getattr(self, "_ws", None) is None:
            import torch
            from bitmask_speculation_b200 import _native
            nbytes = int(_native.library().bms_workspace_bytes(self.device.index))
            self._ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        return self._ws.data_ptr(), self._ws.numel()

    def _alloc_outputs(self):
        import torch
        d = self.device
        r = self.rows
        self.row_tokens = torch.empty(r, dtype=torch.int64, device=d)
        self.row_counts = torch.empty(r, dtype=torch.int64, device=d)
        self.row_status = torch.empty(r, dtype=torch.int32, device=d)
        self.row_budget = torch.empty(r, dtype=torch.int32, device=d)
        if self.kind in ("verify", "grammar"):
            s = self.proposals.shape[0]
            self.accept = torch.empty(s, dtype=torch.int32, device=d)
            self.token = torch.empty(s, dtype=torch.int64, device=d)
            self.kindout = torch.empty(s, dtype=torch.int32, device=d)
            self.seq_status = torch.empty(s, dtype=torch.int32, device=d)

    def _batch(self):
        if self.batches == 1 and hasattr(self, "logits"):
            return self.logits, self.masks
        b = self.step_index % self.batches
        r0 = b * self.rows
        return self.logits_all[r0:r0 + self.rows], self.masks_all[r0:r0 + self.rows]

    def launches_per_step(self):
        return 2 if self.kind in ("verify", "grammar", "vocab") else 1

    def step(self, stream_handle):
        """One hot-path step through the C ABI on inputs resident in HBM."""
        import ctypes
        from bitmask_speculation_b200 import _native
        lib = _native.library()
        dev = self.device.index
        logits, masks = self._batch()
        self.step_index += 1
        if self.kind in ("verify", "grammar"):
            s, k = self.proposals.shape
            rc = lib.bms_verify_batch(
                logits.data_ptr(), 1, masks.data_ptr(), s, k + 1, self.vocab, self.proposals.data_ptr(),
                self.lengths.data_ptr(), ctypes.byref(self.policy), self.row_tokens.data_ptr(),
                self.row_counts.data_ptr(), self.row_status.data_ptr(), self.row_budget.data_ptr(),
                self.accept.data_ptr(), self.token.data_ptr(), self.kindout.data_ptr(),
                self.seq_status.data_ptr(), None, 0, *self.workspace(), dev, stream_handle)
        elif self.kind == "vocab":
            from bitmask_speculation_b200.sharding import vocab_sharded_select
            # Exchange statuses are checked once after the timed loop, not per step.
            self.row_tokens, self.row_counts, self.row_status = vocab_sharded_select(
                logits, masks, self.vocab, exchange=self.exchange, check_exchange=False)
            return
        elif self.kind == "sample":
            b = (self.step_index - 1) % self.batches
            u = self.uniforms_all[b * self.rows:(b + 1) * self.rows]
            rc = lib.bms_masked_sample_batch(
                logits.data_ptr(), self.dtype_code, masks.data_ptr(), self.rows, self.vocab, self.temperature,
                u.data_ptr(), self.row_tokens.data_ptr(), self.row_counts.data_ptr(), self.row_status.data_ptr(),
                *self.workspace(), dev, stream_handle)
        else:
            rc = lib.bms_masked_reduce_batch(
                logits.data_ptr(), self.dtype_code, masks.data_ptr(), self.rows, self.vocab,
                self.row_tokens.data_ptr(), self.row_counts.data_ptr(), self.row_status.data_ptr(),
                *self.workspace(), dev, stream_handle)
        _native.check(rc)

    def kernel_only(self, stream_handle):
        """The dominant kernel alone (fused masked argmax + count, or the sampler)."""
        from bitmask_speculation_b200 import _native
        lib = _native.library()
        logits, masks = self._batch()
        self.step_index += 1
        if self.kind == "sample":
            b = (self.step_index - 1) % self.batches
            u = self.uniforms_all[b * self.rows:(b + 1) * self.rows]
            rc = lib.bms_masked_sample_batch(
                logits.data_ptr(), self.dtype_code, masks.data_ptr(), self.rows, self.vocab, self.temperature,
                u.data_ptr(), self.row_tokens.data_ptr(), self.row_counts.data_ptr(), self.row_status.data_ptr(),
                *self.workspace(), self.device.index, stream_handle)
        elif self.kind == "vocab":
            from bitmask_speculation_b200.sharding import NativeShardBackend
            self._parts = NativeShardBackend().partials(logits, masks, self._offset(), 0.0)
            return
        else:
            rc = lib.bms_masked_reduce_batch(
                logits.data_ptr(), self.dtype_code, masks.data_ptr(), self.rows, self.vocab,
                self.row_tokens.data_ptr(), self.row_counts.data_ptr(), self.row_status.data_ptr(),
                *self.workspace(), self.device.index, stream_handle)
        _native.check(rc)

    def _offset(self):
        from bitmask_speculation_b200.sharding import shard_bounds
        import torch.distributed as dist
        rank = dist.get_rank() if dist.is_initialized() else 0
        return shard_bounds(self.vocab, self.world)[rank][0]

    def check_against_oracle(self):
        """Untimed check of one step against the CPU oracle on every row of the batch: tokens,
        counts and statuses; for verification rounds also the budgets and every per-sequence
        output (accepted length, token, kind, status); for the sampler the tokens within the
        1e-6 CDF-boundary tolerance.  The vocabulary-sharded workload is checked by its tests."""
        import numpy as np
        import torch
        import oracle
        if self.kind == "vocab":
            return
        self.step_index = 0
        logits, masks = self._batch()
        self.step(self.stream_handle())
        torch.cuda.synchronize(self.device)
        self.step_index = 0
        dt = {"bf16": "bfloat16", "f16": "float16", "f32": None}[self.dtype]

        def host(r0, r1):  # a slice of the batch in the oracle's format (bounded host memory)
            part = logits[r0:r1].cpu()
            return (part.view(torch.int16).numpy().view(np.uint16) if dt else part.numpy()), masks[r0:r1].cpu().numpy()

        def same(name, got, want):
            got = got.cpu().numpy() if hasattr(got, "cpu") else np.asarray(got)
            bad = np.flatnonzero(got != want)
            if bad.size:
                raise SystemExit(f"benchmark output {name} differs from the oracle in {bad.size} rows "
                                 f"(first {bad[:4].tolist()})")
        if self.kind == "sample":
            vals, m = host(0, self.rows)
            u = self.uniforms_all[:self.rows].cpu().numpy()
            tok, st = oracle.sample_rows(vals, m, self.temperature, u, dtype=dt)
            same("status", self.row_status, st)
            got = self.row_tokens.cpu().numpy()
            for r in np.flatnonzero(got != tok):
                row = oracle.widen(vals[r], dt) if dt else vals[r]
                if not oracle.sample_matches(row, m[r], self.temperature, u[r], int(got[r]), int(tok[r])):
                    raise SystemExit(f"benchmark sampler row {r} differs from the oracle beyond tolerance")
            return
        parts = [oracle.reduce_rows(*host(r0, min(self.rows, r0 + 4096)), dtype=dt) for r0 in range(0, self.rows, 4096)]
        tok, cnt, st = (np.concatenate([p[i] for p in parts]) for i in range(3))
        same("tokens", self.row_tokens, tok)
        same("counts", self.row_counts, cnt)
        same("status", self.row_status, st)
        if self.kind in ("verify", "grammar"):
            acc, token, kind, sst = oracle.verify(tok, st, self.proposals.cpu().numpy(), self.lengths.cpu().numpy())
            _, budget = oracle.budget_rows(cnt, self.vocab)
            same("row_budget", self.row_budget, budget)
            same("accept_len", self.accept, acc)
            same("token", self.token, token)
            same("kind", self.kindout, kind)
            same("seq_status", self.seq_status, sst)

    def stream_handle(self):
        import torch
        return torch.cuda.current_stream(self.device).cuda_stream


# ---------------------------------------------------------------- e2e through the public API
class EndToEnd:
    """Verification through ``verification.verify_batch`` with host masks/drafts each step."""

    def __init__(self, w: Workload):
        import torch
        self.w = w
        if w.kind == "grammar":
            from bitmask_speculation_b200.grammar_verification import DeviceMaskTable, DraftForkMasks
            s, k = w.proposals.shape
            self.k = k
            self.buf = DraftForkMasks(w.vocab, w.rows, w.device)
            # Device-resident masks: the grammars' state masks live on the device; a round uploads
            # one int32 table index per row.  ``use_table = False`` uploads every row's mask words.
            self.table = DeviceMaskTable.for_grammar(w.grammars[0], w.rows, w.device)
            self.use_table = True
            self.h2d = w.rows * 4 + s * k * 8 + s * 4
            self.h2d_masks = w.rows * w.words * 4 + s * k * 8 + s * 4
            self.d2h = w.rows * (8 + 8 + 4 + 4) + s * (4 + 8 + 4 + 4)
        elif w.kind == "verify":
            from bitmask_speculation_b200.compressed_masks import CompressedMasks
            # The round's masks in their compact transfer form: each row as the smallest of a bitmap,
            # a token-ID list (the enumeration rows) or a byte-coded gap stream (the 5 % rows),
            # expanded on the device into a mask table read through per-row indices.
            self.cm = CompressedMasks.from_bitmaps(w.masks.cpu().numpy(), w.vocab)
            self.tables = [self.cm.allocate(w.device) for _ in range(2)]
            self.h_prop = w.proposals.cpu().pin_memory()
            self.h_len = w.lengths.cpu().pin_memory()
            # Two device input sets and a copy stream: step i's inputs upload while step i-1's
            # kernels run (an engine prefetching the next round's masks); every step still copies
            # its own inputs and reads its own results.
            self.d_prop = [torch.empty_like(w.proposals) for _ in range(2)]
            self.d_len = [torch.empty_like(w.lengths) for _ in range(2)]
            self.copy_stream = torch.cuda.Stream(w.device)
            self.ready = [torch.cuda.Event() for _ in range(2)]
            self.consumed = [torch.cuda.Event() for _ in range(2)]
            for e in self.consumed:
                e.record(torch.cuda.current_stream(w.device))
            self.i = 0
            s = w.proposals.shape[0]
            self.h_out = {
                "accept_len": torch.empty(s, dtype=torch.int32).pin_memory(),
                "token": torch.empty(s, dtype=torch.int64).pin_memory(),
                "kind": torch.empty(s, dtype=torch.int32).pin_memory(),
                "seq_status": torch.empty(s, dtype=torch.int32).pin_memory(),
                "row_budget": torch.empty(w.rows, dtype=torch.int32).pin_memory(),
            }
            self.h2d = self.cm.h2d_bytes + self.h_prop.numel() * 8 + self.h_len.numel() * 4
            self.h2d_bitmaps = w.masks.numel() * 4 + self.h_prop.numel() * 8 + self.h_len.numel() * 4
            self.d2h = sum(t.numel() * t.element_size() for t in self.h_out.values())
        else:
            logits, masks = w._batch()
            self.h_masks = masks.cpu().pin_memory()
            self.d_masks = torch.empty_like(masks)
            self.h_out = {"token": torch.empty(w.rows, dtype=torch.int64).pin_memory(),
                          "status": torch.empty(w.rows, dtype=torch.int32).pin_memory()}
            self.h2d = self.h_masks.numel() * 4
            self.d2h = sum(t.numel() * t.element_size() for t in self.h_out.values())

    def step(self):
        w = self.w
        if w.kind == "grammar":
            # The whole round through the public API: fork masks filled on the host, one H2D, one
            # launch pair, one sync, events replayed on fresh forks of the committed grammars.
            from bitmask_speculation_b200.grammar_verification import verify_with_grammars
            its = verify_with_grammars(w.drafts, w.logits, [g.fork() for g in w.grammars], k=self.k,
                                       buffer=self.buf, table=self.table if self.use_table else None)
            self.events = sum(len(list(it)) for it in its)
        elif w.kind == "verify":
            import torch
            from bitmask_speculation_b200.verification import verify_batch
            b = self.i % 2
            self.i += 1
            compute = torch.cuda.current_stream(w.device)
            with torch.cuda.stream(self.copy_stream):
                self.copy_stream.wait_event(self.consumed[b])  # the kernels that read buffer b are done
                self.d_prop[b].copy_(self.h_prop, non_blocking=True)
                self.d_len[b].copy_(self.h_len, non_blocking=True)
            # Mask bitmaps and ID lists on the copy stream; the list expansion on the compute stream.
            table, mask_rows = self.cm.upload(w.device, self.tables[b], copy_stream=self.copy_stream)
            out = verify_batch(w.logits, table, self.d_prop[b], self.d_len[b], mask_rows=mask_rows)
            self.consumed[b].record(compute)
            for k, h in self.h_out.items():
                h.copy_(getattr(out, k), non_blocking=True)
        else:
            from bitmask_speculation_b200.kernels import cuda
            logits, _ = w._batch()
            self.d_masks.copy_(self.h_masks, non_blocking=True)
            if w.kind == "sample":
                import torch
                u = torch.rand(w.rows, dtype=torch.float64, device=w.device)
                res = cuda.batched_masked_sample(logits, self.d_masks, temperature=w.temperature, uniforms=u)
            else:
                res = cuda.batched_masked_reduce(logits, self.d_masks)
            self.h_out["token"].copy_(res.token_ids, non_blocking=True)
            self.h_out["status"].copy_(res.status, non_blocking=True)


# ---------------------------------------------------------------- timing helpers
def timed_loop(fn, n, device, dist=None):
    """Device time (seconds) of n calls, events on the current stream, max over ranks."""
    import torch
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(device)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(device)
    start.record(stream)
    for _ in range(n):
        fn()
    end.record(stream)
    torch.cuda.synchronize(device)
    seconds = start.elapsed_time(end) / 1e3
    if dist is not None:
        t = torch.tensor([seconds], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        seconds = float(t.item())
        dist.barrier()
    return seconds


def cpu_baseline_grammar(w: Workload, budget_s=10.0):
    """The reference's lazy per-row loop restated on the oracle (one masked argmax per consumed
    row, the grammar advanced in turn) over whole sequences of the round, for ~budget_s seconds;
    rows/s counts the round's K+1 rows per sequence, like the device path."""
    import numpy as np
    import torch
    import oracle
    k = w.proposals.shape[1]
    bits = w.logits.cpu().view(torch.int16).numpy().view(np.uint16)
    seqs = len(w.drafts)
    t0 = time.perf_counter()
    done = 0
    while time.perf_counter() - t0 < budget_s:
        s = done % seqs
        rows = bits[s * (k + 1): s * (k + 1) + len(w.drafts[s]) + 1]
        if not w.grammars[s].is_terminated():
            oracle.grammar_choices(w.drafts[s], rows, w.grammars[s].fork(), dtype="bfloat16")
        done += 1
    elapsed = time.perf_counter() - t0
    return done * (k + 1) / elapsed, 1, f"{done} sequences of the round (reference loop, one thread)"


def cpu_baseline_verify(w: Workload, budget_s=8.0):
    """The CPU oracle (reference algorithm) on this host: reduce + verify + budgets."""
    import numpy as np
    import torch
    import oracle
    threads = host_threads()
    host_logits = w.logits.cpu().view(torch.int16).numpy().view(np.uint16)
    host_masks = w.masks.cpu().numpy()
    proposals = w.proposals.cpu().numpy()
    lengths = w.lengths.cpu().numpy()
    rows = 0
    t0 = time.perf_counter()
    passes = 0
    while True:
        tok, cnt, st = oracle.reduce_rows(host_logits, host_masks, dtype="bfloat16", threads=threads)
        oracle.verify(tok, st, proposals, lengths)
        oracle.budget_rows(cnt, w.vocab)
        rows += host_logits.shape[0]
        passes += 1
        if time.perf_counter() - t0 >= budget_s or passes >= 50:
            break
    elapsed = time.perf_counter() - t0
    return rows / elapsed, threads, f"{passes} full verification rounds ({host_logits.shape[0]} rows each)"


def cpu_baseline_rows(w: Workload, budget_s=8.0):
    import numpy as np
    import torch
    import oracle
    threads = host_threads()
    logits, masks = w._batch()
    if w.dtype == "f32":
        vals, dt = logits.cpu().numpy(), None
    else:
        vals = logits.cpu().view(torch.int16).numpy().view(np.uint16)
        dt = "float16" if w.dtype == "f16" else "bfloat16"
    m = masks.cpu().numpy()
    rows, passes = 0, 0
    t0 = time.perf_counter()
    while True:
        if w.kind == "sample":
            oracle.sample_rows(vals, m, w.temperature, np.random.default_rng(passes).random(w.rows), dtype=dt,
                               threads=threads)
        else:
            oracle.reduce_rows(vals, m, dtype=dt, threads=threads)
        rows += w.rows
        passes += 1
        if time.perf_counter() - t0 >= budget_s or passes >= 2000:
            break
    return rows / (time.perf_counter() - t0), threads, f"{passes} batches of {w.rows} rows"


# ---------------------------------------------------------------- arms
def bench_config(w: Workload, world: int) -> dict:
    """The workload description both arms print (identical for the same arguments)."""
    return {"workload": w.name, "rows_per_gpu": w.rows, "vocab": w.vocab, "bytes_per_row": w.bytes_per_row,
            "l2": (f"inputs {w.rows * w.bytes_per_row * w.batches / 1e9:.2f} GB per GPU rotated "
                   f"({w.batches} batch(es)) > 126 MB L2; no flush"),
            "parallelism": (f"vocab-sharded x{world}, {w.transport}" if w.kind == "vocab"
                            else f"row-sharded x{world}, no collective")}


def sampler_roofline(args, device, peak, peak_kind, rows_list=(64, 256, 2304)):
    """The masked sampler alone at small and large batches (configuration-2 rows tiled, fp16,
    T = 0.7, fresh uniforms; buffers rotated beyond L2): per-launch time and HBM fraction.  At 64
    rows the library takes the flat schedule (two launches), at 256 the fixed one, at 2,304 the
    dynamic one."""
    import copy
    out = {}
    for rows in rows_list:
        a = copy.copy(args)
        a.workload, a.sample_rows, a.sample_density, a.sample_dtype = "sample", rows, None, "float16"
        w = Workload(a, 0, device)
        stream = w.stream_handle()
        probe = timed_loop(lambda: w.kernel_only(stream), 3, device)
        reps = max(20, int(0.75 / max(probe / 3, 1e-6)))
        ktime = timed_loop(lambda: w.kernel_only(stream), reps, device)
        kernel_s = ktime / reps
        achieved = w.rows * w.bytes_per_row / kernel_s / 1e9
        out[str(rows)] = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                          "frac": achieved / peak, "peak_kind": peak_kind, "kernel_us": kernel_s * 1e6,
                          "bytes_per_launch": w.rows * w.bytes_per_row, "launches": reps,
                          "workload": w.name, "l2": f"{w.batches} rotated batches of {w.rows * w.bytes_per_row / 1e6:.0f} MB"}
        del w
    return out


def run_reference_arm(args):
    """The reference algorithm on the host cores (oracle port, all threads), rank 0 only."""
    rank, world, local = dist_env()
    if rank != 0:
        return
    import torch
    import numpy as np
    import oracle
    device = torch.device("cuda", local) if torch.cuda.is_available() else None
    if device is not None:
        torch.cuda.set_device(device)
    threads = host_threads()
    w = Workload(args, 0, device)
    if args.workload == "grammar":
        k = w.proposals.shape[1]
        bits = w.logits.cpu().view(torch.int16).numpy().view(np.uint16)

        def step():
            # Every sequence of the round through the reference's lazy loop, sequences spread
            # over the host threads (each loop is sequential in its rows).
            from concurrent.futures import ThreadPoolExecutor

            def one(s):
                rows = bits[s * (k + 1): s * (k + 1) + len(w.drafts[s]) + 1]
                if not w.grammars[s].is_terminated():
                    oracle.grammar_choices(w.drafts[s], rows, w.grammars[s].fork(), dtype="bfloat16")
            with ThreadPoolExecutor(threads) as ex:
                list(ex.map(one, range(len(w.drafts))))
        rows_per_step = w.rows
        sample = f"full grammar verification round ({len(w.drafts)} sequences, {rows_per_step} rows) per step"
    elif args.workload == "verify":
        host_logits = w.logits.cpu().view(torch.int16).numpy().view(np.uint16)
        host_masks = w.masks.cpu().numpy()
        props, lens = w.proposals.cpu().numpy(), w.lengths.cpu().numpy()

        def step():
            tok, cnt, st = oracle.reduce_rows(host_logits, host_masks, dtype="bfloat16", threads=threads)
            oracle.verify(tok, st, props, lens)
            oracle.budget_rows(cnt, w.vocab)
        rows_per_step = host_logits.shape[0]
        sample = f"full verification round ({rows_per_step} rows) per step"
    else:
        logits, masks = w._batch()
        dt = {"f32": None, "bf16": "bfloat16", "f16": "float16"}[w.dtype]
        vals = logits.cpu().numpy() if dt is None else logits.cpu().view(torch.int16).numpy().view(np.uint16)
        m = masks.cpu().numpy()

        def step():
            if w.kind == "sample":
                oracle.sample_rows(vals, m, w.temperature, np.random.default_rng(0).random(w.rows), dtype=dt,
                                   threads=threads)
            else:
                oracle.reduce_rows(vals, m, dtype=dt, threads=threads)
        rows_per_step = w.rows
        sample = f"{rows_per_step} rows per step"
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    elapsed = time.perf_counter() - t0
    value = rows_per_step * args.steps / elapsed
    port = ("oracle/oracle.c: the reference's CPU algorithm for the path restated in C (torch_reduce, "
            "verify_prefix, DensityPolicy.budget; masked_sample_reference for sampling), OpenMP over "
            f"{threads} host threads. The reference's own PyTorch/Python CPU path is slower than this port "
            "(torch_reduce 508 rows/s on 8 threads at 64 bf16 rows), so ratios against it are conservative.")
    line = {
        "impl": "reference", "metric": "rows/s", "value": value, "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong" if w.kind == "vocab" else "weak", "vs_baseline": None,
        "dtype": w.dtype, "data": "synthetic (seeded, generated on device)", "config": bench_config(w, world),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port", "sample": sample,
                         "implementation": port},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_b200_arm(args):
    import torch
    rank, world, local = dist_env()
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist_mod
        torch.cuda.set_device(local)
        dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
        dist = dist_mod
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    w = Workload(args, rank, device)
    if args.cluster or args.clusters:
        from bitmask_speculation_b200 import _native
        _native.set_launch_override(args.cluster, args.clusters)
    torch.cuda.synchronize(device)
    w.check_against_oracle()
    stream = w.stream_handle()
    peak, peak_kind = measured_peak()

    with ClockSampler(local) as clocks:
        for _ in range(max(3, args.warmup)):
            w.step(stream)
        torch.cuda.synchronize(device)
        torch.cuda.nvtx.range_push("timed")
        seconds = timed_loop(lambda: w.step(stream), args.steps, device, dist)
        torch.cuda.nvtx.range_pop()
        # Dominant kernel alone, long enough (>= roofline_seconds) for the clock samples.
        probe = timed_loop(lambda: w.kernel_only(stream), 3, device)
        reps = max(args.steps, int(args.roofline_seconds / max(probe / 3, 1e-6)))
        torch.cuda.nvtx.range_push("roofline")
        ktime = timed_loop(lambda: w.kernel_only(stream), reps, device)
        torch.cuda.nvtx.range_pop()
        e2e = None
        if not args.no_e2e and w.kind != "vocab":
            e = EndToEnd(w)
            for _ in range(3):
                e.step()
            torch.cuda.synchronize(device)
            if dist is not None:
                dist.barrier()
            # At least 50 end-to-end steps (about a millisecond each): host-link timings vary more
            # than kernel timings.
            esteps = max(args.steps, 50)
            t0 = time.perf_counter()
            torch.cuda.nvtx.range_push("e2e")
            etime = timed_loop(e.step, esteps, device, dist)
            torch.cuda.nvtx.range_pop()
            wall = time.perf_counter() - t0
            if w.kind == "grammar":  # the same round uploading every row's mask words instead
                e.use_table = False
                e.step()
                mtime = timed_loop(e.step, esteps, device, dist)
                e.use_table = True
                uploaded = {"value": w.rows * world * esteps / mtime, "unit": "rows/s",
                            "h2d_bytes_per_step": e.h2d_masks, "d2h_bytes_per_step": e.d2h,
                            "path": "verify_with_grammars with fork masks filled on the host and uploaded"}
            e2e = {"value": w.rows * world * esteps / etime, "unit": "rows/s", "steps": esteps,
                   "h2d_bytes_per_step": e.h2d, "d2h_bytes_per_step": e.d2h,
                   "h2d_bytes_as_bitmaps": getattr(e, "h2d_bitmaps", None),
                   "wall_value": w.rows * world * esteps / wall,
                   "path": {
                       "grammar": ("grammar_verification.verify_with_grammars (public API) with a device-resident "
                                   "mask table: fork state indices computed on the host, one H2D of 4 bytes per "
                                   "row, one launch pair, one sync, events replayed on the sequences' grammars "
                                   "every step"),
                       "verify": ("compressed_masks.CompressedMasks.upload + verification.verify_batch (public API): "
                                  "every step the round's masks go host->device in compact form (each row as the "
                                  "smallest of a bitmap, a token-ID list or a byte-coded gap stream, lists and streams "
                                  "expanded on the device by bms_expand_token_lists / bms_expand_token_gaps) with the "
                                  "drafts and lengths, "
                                  "device-resident logits, results D2H; each step's upload on a copy stream "
                                  "overlaps the previous step's kernels (two input buffers)"),
                       "sample": ("kernels.cuda.batched_masked_sample (public API): pinned host masks H2D, "
                                  "device-resident logits, uniforms drawn on the device, tokens and status D2H "
                                  "every step"),
                   }.get(w.kind, "kernels.cuda.batched_masked_reduce (public API): pinned host masks H2D, "
                                 "device-resident logits, tokens and status D2H every step")}

    sampler = None
    if w.kind == "verify" and world == 1 and not args.no_sampler_roofline:
        with ClockSampler(local) as sclocks:
            sampler = sampler_roofline(args, device, peak, peak_kind)
        sampler["clocks"] = sclocks.summary()
    if w.kind == "vocab" and w.exchange is not None:
        w.exchange.check_statuses(w.row_status)
    total_rows = w.rows if w.kind == "vocab" else w.rows * world  # vocab shards split the same rows
    value = total_rows * args.steps / seconds
    bytes_per_launch = w.rows * w.bytes_per_row
    kernel_s = ktime / reps
    achieved = bytes_per_launch / kernel_s / 1e9
    per_row = NCU_TRAFFIC_PER_ROW.get(w.kind)
    traffic = None if per_row is None else per_row * w.rows
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": "rows/s", "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": seconds / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong" if w.kind == "vocab" else "weak", "vs_baseline": None, "dtype": w.dtype,
        "data": "synthetic (seeded, generated on device)",
        "config": bench_config(w, world),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                     "kernel": "select_rows_kernel (masked argmax + count)" if w.kind != "sample"
                     else "select_rows_kernel (masked sampler)",
                     "kernel_us": kernel_s * 1e6, "bytes_per_launch": bytes_per_launch,
                     "cluster": args.cluster or "auto"},
        "gpu_launches": args.steps * w.launches_per_step(),
        "clocks": clocks.summary(),
    }
    if sampler is not None:
        line["roofline_sampler"] = sampler
    if e2e is not None:
        line["e2e"] = e2e
        if w.kind == "grammar":
            line["e2e_uploaded_masks"] = uploaded
    if not args.no_cpu_baseline and world == 1:
        if w.kind == "grammar":
            v, cores, sample = cpu_baseline_grammar(w)
        elif w.kind == "verify":
            v, cores, sample = cpu_baseline_verify(w)
        else:
            v, cores, sample = cpu_baseline_rows(w)
        line["cpu_baseline"] = {"value": v, "unit": "rows/s", "cores": cores, "kind": "port", "sample": sample}
    print(json.dumps(line), flush=True)


def run_decode(args):
    """End-to-end constrained decoding (the end-to-end configuration): random-init Qwen-style target
    (4 layers, d=1024, 16 heads) and draft (1 layer, d=512), V=248,320 bf16, a 64-state token DFA
    grammar per prompt, ``--prompts`` prompts of 64 random tokens, ``--new-tokens`` tokens each.
    Speculative c4 decoding (density-scheduled K, constrained drafts, batched verification) against
    target-only constrained greedy decoding of the same prompts; outputs must agree token for token.
    """
    import torch
    from bitmask_speculation_b200 import workloads as wl
    from bitmask_speculation_b200.decode import config_models, constrained_greedy, random_prompts, speculative_c4
    rank, world, local = dist_env()
    if rank != 0:
        return
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from bitmask_speculation_b200.grammar_verification import DeviceMaskTable
    vocab = wl.VOCAB
    target, draft = config_models(vocab, device=device)
    prompts = random_prompts(args.prompts, 64, vocab, seed=4)
    grammar0 = wl.SyntheticDFAGrammar(vocab, states=64, seed=4)
    table = DeviceMaskTable.for_grammar(grammar0, 16, device)  # the grammar's state masks on the device
    # warm-up over every padded sequence length the timed runs reach (kernels, cuBLAS heuristics)
    speculative_c4(target, draft, prompts[0], grammar0.fork(), max_new_tokens=args.new_tokens, eos=(0,), table=table)
    speculative_c4(target, draft, prompts[0], grammar0.fork(), max_new_tokens=args.new_tokens, eos=(0,),
                   verify="lazy", table=table)
    constrained_greedy(target, prompts[0], grammar0.fork(), max_new_tokens=args.new_tokens, eos=(0,), table=table)
    torch.cuda.synchronize(device)

    def run(fn, *extra):
        outs = []
        with ClockSampler(local) as clocks:
            t0 = time.perf_counter()
            for p in prompts:
                outs.append(fn(target, *extra, p, grammar0.fork(), max_new_tokens=args.new_tokens, eos=(0,),
                               table=table))
            torch.cuda.synchronize(device)
            secs = time.perf_counter() - t0
        return outs, secs, clocks.summary()

    eager, eager_s, _ = run(speculative_c4, draft)
    lazy, lazy_s, _ = run(lambda *a, **k: speculative_c4(*a, verify="lazy", **k), draft)
    greedy, greedy_s, _ = run(constrained_greedy)
    # The same decoding with each model's embedding and blocks replayed from CUDA graphs (one per
    # padded length, captured by the warm-up).
    target.enable_graphs()
    draft.enable_graphs()
    speculative_c4(target, draft, prompts[0], grammar0.fork(), max_new_tokens=args.new_tokens, eos=(0,), table=table)
    constrained_greedy(target, prompts[0], grammar0.fork(), max_new_tokens=args.new_tokens, eos=(0,), table=table)
    torch.cuda.synchronize(device)
    spec, spec_s, clocks = run(speculative_c4, draft)
    greedy_g, greedy_g_s, _ = run(constrained_greedy)
    tokens = sum(len(o.token_ids) for o in spec)

    def same(x, y):
        return all(a.token_ids == b.token_ids and a.stop_reason == b.stop_reason for a, b in zip(x, y))
    line = {
        "metric": "tokens/s", "value": tokens / spec_s, "unit": "tokens/s", "n_gpus": 1,
        "steps": len(prompts), "warmup": 1, "ms_per_step": spec_s / len(prompts) * 1e3, "higher_is_better": True,
        "scaling": "none", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights, random prompts, synthetic DFA grammar)",
        "config": {"workload": (f"decode: c4 speculative decoding, {len(prompts)} prompts x 64 random tokens, "
                                f"{args.new_tokens} new tokens; target 4 layers d=1024 16 heads, draft 1 layer "
                                "d=512, V=248320 bf16 random-init; 64-state token DFA grammar, EOS id 0; "
                                "state masks resident on the device; model trunks replayed from CUDA graphs"),
                   "rounds": sum(o.rounds for o in spec), "proposed": sum(o.proposed for o in spec),
                   "accepted": sum(o.accepted for o in spec), "tokens": tokens,
                   "stop_reasons": {r: sum(o.stop_reason == r for o in spec) for r in ("eos", "grammar", "length")}},
        "selection_share_of_wall": sum(o.select_seconds for o in spec) / spec_s,
        "device_draft_share_of_wall": sum(o.draft_seconds for o in spec) / spec_s,
        "eager_tokens_per_s": sum(len(o.token_ids) for o in eager) / eager_s,
        "identical_to_eager": same(spec, eager),
        "lazy_verification_tokens_per_s": sum(len(o.token_ids) for o in lazy) / lazy_s,
        "lazy_selection_share_of_wall": sum(o.select_seconds for o in lazy) / lazy_s,
        "identical_to_lazy_verification": same(eager, lazy),
        "greedy_tokens_per_s": sum(len(o.token_ids) for o in greedy_g) / greedy_g_s,
        "eager_greedy_tokens_per_s": sum(len(o.token_ids) for o in greedy) / greedy_s,
        "identical_to_greedy": same(spec, greedy_g),
        "note": ("value: c4 with CUDA-graph model trunks; eager = the same without graphs (must be identical); "
                 "lazy verification = the reference's per-row loop on the same target rows, eager (must be "
                 "identical); greedy = target-only decoding, whose bf16 logits come from forwards of other lengths "
                 "and may differ in near-ties; drafts run on the device (one CUDA graph per draft step: forward, "
                 "masked argmax on the state's table row, DFA step; one read-back per round), so draft selections "
                 "cost no host synchronization: selection_share_of_wall counts the verification calls, "
                 "device_draft_share_of_wall the drafted rounds from launch to read-back"),
        "roofline": None, "clocks": clocks,
        "e2e": {"value": tokens / spec_s, "unit": "tokens/s", "h2d_bytes_per_step": None, "d2h_bytes_per_step": None,
                "path": "decode.speculative_c4 per prompt (host wall clock, model forwards included, graphs)"},
    }
    print(json.dumps(line), flush=True)


def run_stochastic(args):
    """Stochastic speculative acceptance at the verification round's shape: 256 sequences x K = 8
    drafts (``--seqs``), target rows bf16 N(0, 3^2) with the round's masks, draft rows = the target's
    first K rows of each sequence plus N(0, 0.7^2) noise (a close draft model), drafts sampled from
    the draft's masked softmax at T = 0.8 with the batched sampler.  One step = one round through
    ``speculative_accept`` on device-resident inputs: the target and draft rows' sampler partials
    (two selection launches) and the acceptance kernel; rows/s counts the round's target rows.  The
    lazy round (``lazy=True``: one launch normalising only the positions it consumes, up to the
    first rejection) is timed beside it, with the bytes it must read (each consumed position's
    target and draft rows and mask row, then the sampled rows again).  ``--draft-noise`` sets how
    close the draft model is (smaller: longer accepted runs).  No reference implementation exists (the reference's
    contract is greedy), so there is no reference arm; the CPU figure is this rule restated in fp64
    (``oracle.speculative_accept``) on a few sequences."""
    import numpy as np
    import torch
    import oracle
    from bitmask_speculation_b200 import workloads as wl
    from bitmask_speculation_b200.kernels._extension import load_extension
    from bitmask_speculation_b200.stochastic import speculative_accept
    rank, world, local = dist_env()
    if rank != 0:
        return
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    temp, k = 0.8, wl.DRAFT_K
    logits, masks, _, _ = wl.verify_batch_torch(args.seqs, seed=3, device=device)
    seqs, vocab = args.seqs, wl.VOCAB
    words = masks.shape[1]
    g = torch.Generator(device=device).manual_seed(7)
    first_k = logits.view(seqs, k + 1, vocab)[:, :k].reshape(seqs * k, vocab)
    draft = (first_k.float() + args.draft_noise * torch.randn(first_k.shape, generator=g, device=device)).to(
        torch.bfloat16)
    del first_k
    dmasks = masks.view(seqs, k + 1, words)[:, :k].reshape(seqs * k, words).contiguous()
    native = load_extension()
    u = torch.rand(seqs * k, dtype=torch.float64, generator=g, device=device)
    proposals = native.masked_sample_batch(draft, dmasks, temp, u)[0].view(seqs, k).contiguous()
    lengths = torch.full((seqs,), k, dtype=torch.int32, device=device)
    ua = torch.rand((seqs, k), dtype=torch.float64, generator=g, device=device)
    ur = torch.rand(seqs, dtype=torch.float64, generator=g, device=device)

    def step(lazy=False):
        return speculative_accept(logits, draft, masks, proposals, lengths, temperature=temp, accept_uniforms=ua,
                                  resample_uniforms=ur, lazy=lazy)
    out = step()
    # Untimed check against the fp64 restatement on the first sequences.
    n_chk = 6
    tf = (logits[: n_chk * (k + 1)].cpu().view(torch.int16).numpy().view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    df = (draft[: n_chk * k].cpu().view(torch.int16).numpy().view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    want = oracle.speculative_accept(tf, df, masks[: n_chk * (k + 1)].cpu().numpy(), proposals[:n_chk].cpu().numpy(),
                                     lengths[:n_chk].cpu().numpy(), temp, ua[:n_chk].cpu().numpy(), ur[:n_chk].cpu().numpy())
    acc = out.accept_len.cpu().numpy()
    for s_, (j, _, _, margin, _) in enumerate(want):
        if margin > 1e-5 and acc[s_] != j:
            raise SystemExit("stochastic acceptance differs from the restated rule")
    lazy_out = step(lazy=True)
    same = float((lazy_out.accept_len == out.accept_len).logical_and(lazy_out.token == out.token).double().mean().item())
    with ClockSampler(local) as clocks:
        for _ in range(max(3, args.warmup)):
            step()
        torch.cuda.nvtx.range_push("timed")
        seconds = timed_loop(step, args.steps, device)
        torch.cuda.nvtx.range_pop()
        for _ in range(3):
            step(lazy=True)
        seconds_lazy = timed_loop(lambda: step(lazy=True), args.steps, device)
    per_step = seconds / args.steps
    rows = seqs * (k + 1)
    algorithmic = (rows + seqs * k) * (vocab * 2 + words * 4 + 32) + seqs * 2 * vocab * 2
    # Bytes the lazy launch reads: positions 0..j of each sequence (target row, mask row, and the
    # draft row below L), then the sampled target row, its mask row and, for a replacement, the
    # draft row again.
    row_b, mask_b = vocab * 2, words * 4
    jj, ll = acc.astype(np.int64), lengths.cpu().numpy().astype(np.int64)
    lazy_bytes = int(((jj + 1) * (row_b + mask_b) + np.minimum(jj + 1, ll) * row_b
                      + row_b + mask_b + (jj < ll) * row_b).sum())
    t0 = time.perf_counter()
    oracle.speculative_accept(tf, df, masks[: n_chk * (k + 1)].cpu().numpy(), proposals[:n_chk].cpu().numpy(),
                              lengths[:n_chk].cpu().numpy(), temp, ua[:n_chk].cpu().numpy(), ur[:n_chk].cpu().numpy())
    cpu_rows = n_chk * (k + 1) / (time.perf_counter() - t0)
    peak, peak_kind = measured_peak()
    line = {
        "metric": "rows/s", "value": rows / per_step, "unit": "rows/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, generated on device)",
        "config": {"workload": (f"stochastic: {seqs} sequences x K={k} drafts sampled from a draft model at T={temp} "
                                f"(draft = target + N(0, {args.draft_noise}^2)), V={vocab} bf16, "
                                "verification-round masks; target rows/s"),
                   "rows_per_gpu": rows, "draft_rows": seqs * k},
        "roofline": {"bound": "hbm", "achieved": algorithmic / per_step / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": algorithmic / per_step / 1e9 / peak, "peak_kind": peak_kind,
                     "kernel": "whole step (two sampler-partials launches + acceptance kernel)",
                     "bytes_per_step": algorithmic},
        "lazy": {"ms_per_step": seconds_lazy / args.steps * 1e3, "bytes_per_step": lazy_bytes,
                 "frac": lazy_bytes / (seconds_lazy / args.steps) / 1e9 / peak,
                 "same_accept_len_and_token": same},
        "gpu_launches": 3 * args.steps, "clocks": clocks.summary(),
        "acceptance_rate": float(out.accept_len.double().mean().item()) / k,
        "cpu_baseline": {"value": cpu_rows, "unit": "rows/s", "cores": 1, "kind": "port",
                         "sample": f"{n_chk} sequences through oracle.speculative_accept (fp64 numpy restatement of "
                                   "this library's rule; the reference has no stochastic acceptance)"},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.workload == "stochastic":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference has no stochastic speculative "
                              "acceptance (its correctness contract is greedy, docs/design.md:5-11)"}), flush=True)
        else:
            run_stochastic(args)
        return
    if args.workload == "decode":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference's engine (Transformers models, "
                              "request loop) is outside the rebuilt path; its decoding semantics are restated in "
                              "decode.py and checked against target-only greedy decoding"}), flush=True)
        else:
            run_decode(args)
        return
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_b200_arm(args)


if __name__ == "__main__":
    main()
