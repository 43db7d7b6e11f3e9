"""Model runner: cache pools, batch preparation, eager and CUDA-graph execution,
sampling.

Per step the runner turns a :class:`SchedulerOutput` into the device tensors
of a :class:`StepContext` (one host->device copy per tensor from pinned
buffers), runs the model and the sampler, and copies the sampled token ids
back.  Decode-only batches replay a CUDA graph captured per padded batch size
(the reference's FULL decode graphs, vllm_sm80/worker/graph_mem_worker.py:64):
padding rows point at the reserved KV block 0 and state slot 0 and write
nothing (slot mapping -1).
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass

import numpy as np
import torch

from .. import _ext
from ..config import EngineConfig
from ..models import hybrid
from ..models.hybrid import HybridForCausalLM, StepContext
from ..ops import sampling as sampling_ops
from ..parallel import comm
from ..parallel import state as pstate
from .block_pool import SlotPool, make_block_pool
from .failed_inputs import sanitize, sanitize_dict
from .scheduler import SchedulerOutput


@dataclass
class StepStats:
    num_tokens: int = 0
    graph: bool = False
    h2d_bytes: int = 0
    d2h_bytes: int = 0
    device_ms: float = 0.0


class ModelRunner:
    def __init__(self, cfg: EngineConfig, model: HybridForCausalLM | None = None):
        self.cfg = cfg
        self.st = pstate.get()
        self.device = torch.device(cfg.device if cfg.device != "cuda" else f"cuda:{self.st.local_rank}") \
            if torch.cuda.is_available() and cfg.device.startswith("cuda") else torch.device("cpu")
        self.model = model or HybridForCausalLM(cfg.model, self.device, cfg.seed)
        self.mcfg = cfg.model
        self.block_size = cfg.cache.block_size
        assert self.block_size == 64, "the sparse-MLA kernels use 64-token blocks"
        self.max_blocks_per_seq = math.ceil(cfg.scheduler.max_model_len / self.block_size)
        from .. import envs

        self._check_indices = bool(envs.get("VLLM_B200_STATE_INDEX_CHECK"))
        for _name, src in self._ngram_sources():
            sc = cfg.scheduler
            src.reserve(max(sc.max_num_batched_tokens, sc.max_num_seqs * (1 + sc.num_speculative_tokens)))
        self._alloc_caches()
        self.step_counter = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.graphs: dict[int, tuple] = {}
        self._packed: dict[int, tuple] = {}
        self.spec_graphs: dict[tuple, tuple] = {}
        self._status_h = torch.zeros(1, dtype=torch.int32, pin_memory=torch.cuda.is_available())
        self.graph_pool = None
        self.last_stats = StepStats()
        self.time_device = False  # record CUDA events around each step's device work
        from .. import envs
        from ..utils.light_timing import LightTimer

        self.timer = LightTimer.from_env(self.device)
        if self.timer is not None:
            self.timer.attach(self.model)
        envs.log_gate("light timing", self.timer is not None)
        envs.log_gate("state index check", self._check_indices)
        self.spec = None
        self._pending = None
        self._pp_hidden: list = []
        if cfg.scheduler.num_speculative_tokens > 0 and cfg.scheduler.spec_method == "dflash":
            # every stage keeps the DFlash drafter's auxiliary hidden states of its layers; they travel
            # to the last stage with the pipeline hop
            from ..models.dflash import DFlashConfig

            dc = DFlashConfig(num_layers=cfg.scheduler.dflash_layers).resolve(cfg.model)
            self.model.aux_layer_ids = tuple(dc.aux_layer_ids)
        if cfg.scheduler.num_speculative_tokens > 0 and self.st.is_last_pp:
            from .spec_decode import SpecDecoder

            self.spec = SpecDecoder(self, cfg.scheduler.num_speculative_tokens)

    # ------------------------------------------------------------------ caches
    @torch.no_grad()
    def fill_caches_random(self, seed: int = 0, state_std: float = 0.1) -> None:
        """Benchmarks of long-context decode without a prefill: every latent row ~N(0, 1), index keys
        fp8 codes of N(0, 1) values with unit scales, recurrent KDA states ~N(0, state_std^2), conv windows
        ~N(0, 1) (requests added with a synthetic prefix then attend to these rows)."""
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        for lat, idx_k, idx_s in self.mla_caches.values():
            lat.normal_(generator=g)
            idx_k.copy_(torch.randn(idx_k.shape, generator=g, device=self.device).to(torch.float8_e4m3fn)
                        .view(torch.uint8))
            idx_s.fill_(1.0)
        for rec, conv in self.kda_states.values():
            rec.normal_(generator=g).mul_(state_std)
            conv.normal_(generator=g)

    def _alloc_caches(self):
        cfg = self.cfg
        m = self.model
        kda_ids, mla_ids = m.kda_layer_ids(), m.mla_layer_ids()
        self.num_slots = cfg.scheduler.max_num_seqs + 1
        rec_shape, conv_shape = m.kda_state_shapes()
        nb = cfg.cache.num_blocks
        if nb <= 0:
            if self.device.type == "cuda":
                torch.cuda.synchronize()
                free, _total = torch.cuda.mem_get_info(self.device)
                kda_bytes = len(kda_ids) * self.num_slots * (math.prod(rec_shape) * 4 + math.prod(conv_shape) * 2)
                spec = cfg.scheduler.num_speculative_tokens > 0
                mtp = spec and cfg.scheduler.spec_method == "mtp"
                mtp_gqa = mtp and "mla" not in self.mcfg.layer_types and "gqa" in self.mcfg.layer_types
                n_mla = len(mla_ids) + (1 if mtp and not mtp_gqa else 0)  # + MTP layer
                per_block = max(1, n_mla) * 64 * (576 * 2 + 128 + 4)
                n_gqa = len(m.gqa_layer_ids()) + (1 if mtp_gqa else 0)
                if n_gqa:  # [k | v] rows of the local key-value heads
                    per_block += n_gqa * 64 * m.gqa_kv_heads() * 512 * 2
                if spec and not mtp:  # DFlash [k | v | 0] rows of 512 per key-value head (the default 4 heads)
                    per_block += cfg.scheduler.dflash_layers * 64 * 4 * 512 * 2
                n_dsa = len(m.dsa_layer_ids())
                if n_dsa:  # DeepSeek-V4.1 group rows + index keys, and the per-slot rings / step scratch
                    a = self.mcfg.dsa
                    per_block += n_dsa * 64 * (a.head_dim * 2 + a.index_head_dim * 2)
                    sc = cfg.scheduler
                    k = sc.num_speculative_tokens
                    kda_bytes += n_dsa * (self.num_slots * ((a.window + k) * a.head_dim * 2 + (k + 2) * a.head_dim * 8)
                                          + max(sc.max_num_batched_tokens, sc.max_num_seqs) * a.head_dim * 2)
                scratch = self._activation_reserve()
                free, _total = torch.cuda.mem_get_info(self.device)
                avail = free * cfg.cache.gpu_memory_utilization - kda_bytes - scratch
                nb = int(max(avail, 0) // per_block)
                want = cfg.scheduler.max_num_seqs * self.max_blocks_per_seq + 1
                nb = max(2, min(nb, want))
            else:
                nb = cfg.scheduler.max_num_seqs * self.max_blocks_per_seq + 1
        self._make_caches(nb)
        self.graphs_ok = True

    def _activation_reserve(self) -> int:
        """Bytes a full prefill step allocates on top of the caches, measured: one forward of
        max_num_batched_tokens prompt tokens (sequences of up to max_model_len tokens, no cache rows
        written) over a cache of one sequence's blocks, the peak of the allocator minus its level before,
        plus a quarter and 1 GiB for CUDA graphs and the drafter (the reference sizes its KV pool from
        a profiling run the same way, vllm_sm80/kv_planning.py:48,503).  With pipeline parallelism (a
        forward needs the other stages) a fixed 6 GiB."""
        from .request import Request, SamplingParams
        from .scheduler import ScheduledReq

        sc = self.cfg.scheduler
        if self.st.pp_size > 1 or self.device.type != "cuda":
            return 6 << 30
        self._make_caches(self.max_blocks_per_seq + 1)
        T = max(sc.max_num_batched_tokens, 1)
        L = max(1, min(sc.max_model_len - 1, T))
        reqs, left = [], T
        while left > 0 and len(reqs) < sc.max_num_seqs:
            n = min(L, left)
            r = Request([1] * n, SamplingParams(max_tokens=1), request_id=f"__profile_{len(reqs)}__")
            r.block_ids = [0] * self.max_blocks_per_seq
            r.kda_slot = 0
            reqs.append(ScheduledReq(r, n, 0, True))
            left -= n
        out = SchedulerOutput(reqs=reqs)
        torch.cuda.synchronize(self.device)
        torch.cuda.reset_peak_memory_stats(self.device)
        base = torch.cuda.memory_allocated(self.device)
        with torch.inference_mode():
            h = self._host_inputs(out)
            h["slots"][:] = -1  # no cache rows written
            dev, ctx, _ = self._context(h)
            hidden = self.model(dev["ids"], ctx)
            self.model.compute_logits(hidden.index_select(0, self._to_dev(h["sample_rows"])))
        torch.cuda.synchronize(self.device)
        peak = torch.cuda.max_memory_allocated(self.device) - base
        del hidden, dev, ctx
        self.mla_caches, self.kda_states, self.dsa_cores, self.gqa_caches = {}, {}, {}, {}
        torch.cuda.empty_cache()
        self.activation_peak = int(peak)
        return int(peak * 1.25) + (1 << 30)

    def _make_caches(self, nb: int) -> None:
        cfg = self.cfg
        m = self.model
        kda_ids, mla_ids = m.kda_layer_ids(), m.mla_layer_ids()
        rec_shape, conv_shape = m.kda_state_shapes()
        self.num_blocks = nb
        rows = nb * 64
        self.mla_caches = {}
        for i in mla_ids:
            self.mla_caches[i] = (torch.zeros(rows, 576, dtype=torch.bfloat16, device=self.device),
                                  torch.zeros(rows, 128, dtype=torch.uint8, device=self.device),
                                  torch.ones(rows, dtype=torch.float32, device=self.device))
        self.kda_states = {}
        for i in kda_ids:
            self.kda_states[i] = (torch.zeros(self.num_slots, *rec_shape, dtype=torch.float32, device=self.device),
                                  torch.zeros(self.num_slots, *conv_shape, dtype=torch.bfloat16, device=self.device))
        # DeepSeek-V4.1 attention: compressed groups paged on the token blocks, a window ring per
        # state slot, one step's window rows of scratch
        self.dsa_cores = {}
        dsa_ids = m.dsa_layer_ids()
        sc = cfg.scheduler
        max_step = max(sc.max_num_batched_tokens, sc.max_num_seqs) * (1 + sc.num_speculative_tokens)
        for i in dsa_ids:
            self.dsa_cores[i] = m.layer(i).attn.make_core(self.num_slots, rows, max_step,
                                                           sc.num_speculative_tokens, self.device)
        self.gqa_caches = {}
        for i in m.gqa_layer_ids():
            self.gqa_caches[i] = torch.zeros(*m.layer(i).attn.cache_rows(rows), dtype=torch.bfloat16,
                                             device=self.device)
        self.block_pool = make_block_pool(nb, 1)
        self.slot_pool = SlotPool(self.num_slots, 1) if (kda_ids or dsa_ids) else None

    # ------------------------------------------------------------------ inputs
    def _bt_row(self, r) -> np.ndarray:
        """The request's block-table row, kept on the request and extended as blocks are appended.  A
        preemption gives the request a new block list (the cached row holds the old list, so its
        identity cannot be reused), which rebuilds the row."""
        row = getattr(r, "_bt_row", None)
        ids = r.block_ids
        n = len(ids)
        if row is None or r._bt_list is not ids or n < r._bt_len:
            row = np.zeros(self.max_blocks_per_seq, dtype=np.int32)
            row[:n] = ids
            r._bt_row, r._bt_list, r._bt_len = row, ids, n
        elif n > r._bt_len:
            row[r._bt_len:n] = ids[r._bt_len:]
            r._bt_len = n
        return row

    def _host_inputs_decode(self, out: SchedulerOutput, Sp: int):
        """_host_inputs of a step where every request computes one token (no drafts), vectorised."""
        reqs = out.reqs
        S = len(reqs)
        a = np.fromiter((s.start for s in reqs), dtype=np.int64, count=S)
        blk = np.fromiter((s.req.block_ids[s.start // 64] for s in reqs), dtype=np.int64, count=S)
        ids = np.zeros(Sp, dtype=np.int64)
        ids[:S] = np.fromiter((s.req.token_at(s.start) for s in reqs), dtype=np.int64, count=S)
        pos = np.zeros(Sp, dtype=np.int32)
        pos[:S] = a
        slots = np.full(Sp, -1, dtype=np.int64)
        slots[:S] = blk * 64 + a % 64
        tseq = np.arange(Sp, dtype=np.int32)
        tseq[S:] = 0
        ctx = np.ones(Sp, dtype=np.int32)
        ctx[:S] = a + 1
        cu = np.arange(Sp + 1, dtype=np.int32)
        kslot = np.zeros(Sp, dtype=np.int32)
        kslot[:S] = np.fromiter((max(s.req.kda_slot, 0) for s in reqs), dtype=np.int32, count=S)
        hinit = np.zeros(Sp, dtype=np.int32)
        hinit[:S] = a > 0
        bt = np.zeros((Sp, self.max_blocks_per_seq), dtype=np.int32)
        if S:
            bt[:S] = np.stack([self._bt_row(s.req) for s in reqs])
        temps = np.zeros(Sp, dtype=np.float32)
        temps[:S] = np.fromiter((s.req.params.temperature for s in reqs), dtype=np.float32, count=S)
        sample_rows = np.fromiter((i for i, s in enumerate(reqs) if s.sample), dtype=np.int64)
        h = dict(ids=ids, pos=pos, slots=slots, tseq=tseq, ctx=ctx, cu=cu, kslot=kslot, hinit=hinit, bt=bt,
                 temps=temps, bans=self._bans_rows(reqs, Sp), sample_rows=sample_rows,
                 max_ctx=int(a.max()) + 1 if S else 1, T=Sp, S=Sp)
        self._add_ngram_ids(h, ((s.req, s.start, 1, 0) for s in reqs), Sp)
        return h

    @staticmethod
    def _bans_rows(reqs, rows: int) -> np.ndarray:
        """[rows, MAX_BANS] banned token ids of each sequence's sampled row (-1 = none)."""
        bans = np.full((rows, sampling_ops.MAX_BANS), -1, dtype=np.int32)
        for i, s in enumerate(reqs):
            b = s.req.params.bad_token_ids
            if b:
                bans[i, :len(b)] = b[:sampling_ops.MAX_BANS]
        return bans

    def _ngram_sources(self) -> list:
        """(input name, source) of the model's n-gram tables: the PLE embedding ("ple") and the Engram
        memory ("engram"); each source has `ids_of(tokens, positions)`, `max_order` and `heads`."""
        out = []
        if getattr(self.model, "ple", None) is not None:
            out.append(("ple", self.model.ple))
        if getattr(self.model, "engram", None) is not None:
            out.append(("engram", self.model.engram))
        return out

    def _add_ngram_ids(self, h: dict, items, rows: int) -> None:
        """n-gram ids [rows, heads] of the step's tokens for every n-gram table of the model, into h:
        items = (request, first position, tokens, drafts among them) per scheduled sequence, in row order;
        padding rows keep id 0."""
        srcs = self._ngram_sources()
        if not srcs:
            return
        items = list(items)
        for name, src in srcs:
            out = np.zeros((rows, src.heads), dtype=np.int64)
            t = 0
            for r, a, n, nd in items:
                w0 = max(0, a - src.max_order + 1)
                toks = r.tokens(w0, a + n - nd) + list(r.draft_token_ids[:nd])
                out[t:t + n] = src.ids_of(toks, np.arange(a - w0, a - w0 + n))
                t += n
            h[name] = out

    def _host_inputs(self, out: SchedulerOutput, pad_to: int | None = None):
        reqs = out.reqs
        S = len(reqs)
        T = out.num_tokens
        if T == S and all(s.num_new == 1 and s.num_draft == 0 for s in reqs) and not self._check_indices:
            return self._host_inputs_decode(out, pad_to or S)
        Sp = pad_to or S
        Tp = T + (Sp - S)  # decode padding: one token per padded sequence
        ids = np.zeros(Tp, dtype=np.int64)
        pos = np.zeros(Tp, dtype=np.int32)
        slots = np.full(Tp, -1, dtype=np.int64)
        tseq = np.zeros(Tp, dtype=np.int32)
        ctx = np.ones(Tp, dtype=np.int32)
        cu = np.zeros(Sp + 1, dtype=np.int32)
        kslot = np.zeros(Sp, dtype=np.int32)
        hinit = np.zeros(Sp, dtype=np.int32)
        bt = np.zeros((Sp, self.max_blocks_per_seq), dtype=np.int32)
        temps = np.zeros(Sp, dtype=np.float32)
        sample_rows = []
        t = 0
        max_ctx = 1
        for i, s in enumerate(reqs):
            r = s.req
            n = s.num_new
            a = s.start
            seq_tokens = r.tokens(a, a + n - s.num_draft) + list(r.draft_token_ids[: s.num_draft])
            ids[t:t + n] = seq_tokens
            p = np.arange(a, a + n, dtype=np.int32)
            pos[t:t + n] = p
            b = np.asarray(r.block_ids, dtype=np.int64)
            slots[t:t + n] = b[p // 64] * 64 + p % 64
            tseq[t:t + n] = i
            ctx[t:t + n] = p + 1
            max_ctx = max(max_ctx, a + n)
            cu[i + 1] = cu[i] + n
            kslot[i] = max(r.kda_slot, 0)
            hinit[i] = 1 if a > 0 else 0
            bt[i] = self._bt_row(r)
            temps[i] = r.params.temperature
            if s.sample:
                if s.num_draft:
                    sample_rows.extend(range(t, t + n))
                else:
                    sample_rows.append(t + n - 1)
            t += n
        for i in range(S, Sp):  # decode padding rows
            cu[i + 1] = cu[i] + 1
        h = dict(ids=ids, pos=pos, slots=slots, tseq=tseq, ctx=ctx, cu=cu, kslot=kslot, hinit=hinit, bt=bt,
                 temps=temps, bans=self._bans_rows(reqs, Sp), sample_rows=np.asarray(sample_rows, dtype=np.int64),
                 max_ctx=max_ctx, T=Tp, S=Sp)
        self._add_ngram_ids(h, ((s.req, s.start, s.num_new, s.num_draft) for s in reqs), Tp)
        if self._check_indices:
            from ..utils.state_check import check_step

            check_step(h, out, self.num_blocks, self.block_size, self.num_slots if self.slot_pool else 0,
                       self.cfg.scheduler.max_model_len)
        return h

    def _to_dev(self, a: np.ndarray, out: torch.Tensor | None = None) -> torch.Tensor:
        t = torch.from_numpy(a)
        if self.device.type == "cuda":
            t = t.pin_memory()
            if out is not None:
                out.copy_(t, non_blocking=True)
                return out
            return t.to(self.device, non_blocking=True)
        if out is not None:
            out.copy_(t)
            return out
        return t

    def _context(self, h: dict, bufs: dict | None = None, max_ctx: int | None = None) -> tuple:
        b = bufs or {}
        keys = ("ids", "pos", "slots", "tseq", "ctx", "cu", "kslot", "hinit", "bt", "temps") + tuple(
            k for k in ("ple", "engram") if k in h)
        dev = {k: self._to_dev(h[k], b.get(k)) for k in keys}
        ctx = StepContext(positions=dev["pos"], num_tokens=h["T"], slot_mapping=dev["slots"], token_seq=dev["tseq"],
                          ctx_lens=dev["ctx"], block_table=dev["bt"], max_ctx=max_ctx or h["max_ctx"],
                          cu_seqlens=dev["cu"], kda_slots=dev["kslot"], has_init=dev["hinit"],
                          dsa_cores=self.dsa_cores, gqa_caches=self.gqa_caches,
                          mla_caches=self.mla_caches, kda_states=self.kda_states,
                          scores_buf=b.get("scores"), ple_ids=dev.get("ple"),
                          engram_ids=dev.get("engram"))
        nbytes = sum(h[k].nbytes for k in keys)
        return dev, ctx, nbytes

    # ------------------------------------------------------------------ forward + sample
    def _forward_sample(self, ids, ctx, sample_rows, temps, seed, bans=None):
        if self.timer is not None:
            self.timer.open_row()
        return self._sample_hidden(self.model(ids, ctx), sample_rows, temps, seed, bans)

    def _sample_hidden(self, hidden, sample_rows, temps, seed, bans=None):
        hs = hidden if sample_rows is None else hidden.index_select(0, sample_rows)
        logits = self.model.compute_logits(hs)
        val, idx = sampling_ops.sample_local(logits, temps, seed, self.step_counter, self.model.vocab_offset, bans)
        if self.st.tp_size > 1:
            vals = comm.tp_all_gather(val[None], dim=0)
            idxs = comm.tp_all_gather(idx[None], dim=0)
            return sampling_ops.combine(vals, idxs)
        return idx.long()

    @torch.inference_mode()
    def _graph_step(self, out: SchedulerOutput) -> bool:
        return (not self.cfg.enforce_eager and self.graphs_ok and self.device.type == "cuda" and out.decode_only
                and all(s.num_draft == 0 for s in out.reqs)
                and len(out.reqs) <= max(self.cfg.cuda_graph_batch_sizes))

    def can_launch(self, out: SchedulerOutput) -> bool:
        """Whether `out` is a decode step that `launch` can queue without the host knowing its input
        tokens (one pipeline stage, no speculative decoding, no n-gram tables hashed on the host)."""
        return (bool(out.reqs) and self.st.pp_size == 1 and self.spec is None and out.decode_only
                and all(s.num_draft == 0 for s in out.reqs) and not self._ngram_sources()
                and len(out.reqs) <= max(self.cfg.cuda_graph_batch_sizes))

    def execute(self, out: SchedulerOutput) -> dict[str, list[int]]:
        if not out.reqs:
            return {}
        if self.st.pp_size > 1:
            return self._execute_pp(out)
        if self.spec is not None:
            return self._execute_spec(out)
        if self._graph_step(out):
            return self.finish(out, self.launch(out))
        stats = StepStats(num_tokens=out.num_tokens, graph=False)
        h = self._host_inputs(out)
        dev, ctx, nbytes = self._context(h)
        rows = self._to_dev(h["sample_rows"])
        temps_rows = self._sample_temps(out, h)
        bans = self._sample_bans(out)
        ev = self._ev_start()
        tokens = self._forward_sample(dev["ids"], ctx, rows, temps_rows, self.cfg.seed, bans)
        self._ev_end(ev)
        return self.finish(out, self._readback(tokens, stats, nbytes))

    def launch(self, out: SchedulerOutput, prev: tuple | None = None) -> dict:
        """Queue one decode step as a graph replay and the read-back of its tokens; returns the handle
        `finish` completes.  prev = (the previous step's output, its handle): tokens the host does not
        know yet (the previous step's, still in flight) are taken on the device from that step's sampled
        tokens, request by request, before the replay (asynchronous scheduling).  Without graphs the step
        runs eagerly the same way."""
        if not self._graph_step(out):
            return self._launch_eager(out, prev)
        B = next(b for b in sorted(self.cfg.cuda_graph_batch_sizes) if b >= len(out.reqs))
        if B not in self.graphs:
            self._capture(B)
        g, bufs, ids_out = self.graphs[B]
        h = self._host_inputs(out, pad_to=B)
        nbytes = self._stage_graph_inputs(B, h)
        if prev is not None:
            # the previous step's sampled tokens (that graph's output buffer, read before this replay
            # overwrites it) gathered into this step's input ids
            src_h = self._gather_rows(out, prev[0], B)
            nbytes += src_h.nbytes
            torch.index_select(prev[1]["tokens_dev"].to(bufs["ids"].dtype), 0, self._to_dev(src_h), out=bufs["ids"])
        ev = self._ev_start()
        g.replay()
        self._ev_end(ev)
        tokens = ids_out[: len(out.reqs)]
        stats = StepStats(num_tokens=out.num_tokens, graph=True)
        return self._readback(tokens, stats, nbytes, keep_dev=ids_out[:B])

    @staticmethod
    def _gather_rows(out: SchedulerOutput, prev_out: SchedulerOutput, rows: int) -> np.ndarray:
        """Row of each of `out`'s requests in `prev_out` (0 for padding rows)."""
        row_of = {s.req.request_id: i for i, s in enumerate(prev_out.reqs)}
        src = np.zeros(rows, dtype=np.int64)
        src[:len(out.reqs)] = [row_of.get(s.req.request_id, 0) for s in out.reqs]
        return src

    def _launch_eager(self, out: SchedulerOutput, prev: tuple | None) -> dict:
        h = self._host_inputs(out)
        dev, ctx, nbytes = self._context(h)
        if prev is not None:
            src = self._to_dev(self._gather_rows(out, prev[0], dev["ids"].shape[0]))
            torch.index_select(prev[1]["tokens_dev"].to(dev["ids"].dtype), 0, src, out=dev["ids"])
        rows = self._to_dev(h["sample_rows"])
        ev = self._ev_start()
        tokens = self._forward_sample(dev["ids"], ctx, rows, self._sample_temps(out, h), self.cfg.seed,
                                      self._sample_bans(out))
        self._ev_end(ev)
        return self._readback(tokens, StepStats(num_tokens=out.num_tokens, graph=False), nbytes, keep_dev=tokens)

    def _readback(self, tokens: torch.Tensor, stats: "StepStats", nbytes: int, keep_dev=None) -> dict:
        """Queue the step's device-to-host token copy (and the status word's) without waiting."""
        self.step_counter += 1
        hnd = {"stats": stats, "nbytes": nbytes, "out_bytes": tokens.numel() * tokens.element_size(),
               "tokens_dev": keep_dev}
        if self.device.type == "cuda":
            # the status word rides on the tokens' read-back: copied first, valid once they arrive
            status = torch.empty(1, dtype=torch.int32, pin_memory=True)
            status.copy_(_ext.status_word(self.device), non_blocking=True)
            host = torch.empty(tokens.shape, dtype=tokens.dtype, pin_memory=True)
            host.copy_(tokens, non_blocking=True)
            done = torch.cuda.Event()
            done.record()
            hnd.update(status=status, host=host, done=done, events=self._events)
            self._events = None
        else:
            hnd.update(host=tokens, events=None)
        return hnd

    def finish(self, out: SchedulerOutput, hnd: dict) -> dict[str, list[int]]:
        """Wait for a launched step's tokens and return them per request."""
        if "done" in hnd:
            hnd["done"].synchronize()
        host = hnd["host"].tolist()
        stats = hnd["stats"]
        if hnd.get("events") is not None:
            a, b = hnd["events"]
            stats.device_ms = a.elapsed_time(b)
        stats.h2d_bytes = hnd["nbytes"]
        stats.d2h_bytes = hnd["out_bytes"]
        self.last_stats = stats
        if self.device.type == "cuda":
            _ext.raise_status(self.device, int(hnd["status"][0]))
        return self._split_tokens(out, sanitize(host, self.mcfg.vocab_size))

    _events = None

    # ------------------------------------------------------------------ pipeline parallel
    def _micro_batches(self, out: SchedulerOutput) -> list[SchedulerOutput]:
        """Split the step into up to pp_size micro-batches, so stage s works on micro-batch i + 1 while
        stage s + 1 works on i.  With decode spreading (the reference's PP decode cap,
        vllm_sm80/sched/scheduler.py:329) every micro-batch takes an equal share of the decoding
        requests and the prefill chunks fill in by token count, so no micro-batch holds all the decodes
        behind a long chunk; otherwise consecutive requests with about equal token counts."""
        n = min(self.st.pp_size, len(out.reqs))
        if self.cfg.scheduler.pp_spread_decodes and n > 1:
            bins = [[] for _ in range(n)]
            load = [0] * n
            decodes = [s for s in out.reqs if s.num_new - s.num_draft == 1 and s.start > 0]
            did = {id(s) for s in decodes}
            for j, s in enumerate(decodes):
                bins[j % n].append(s)
                load[j % n] += s.num_new
            for s in sorted((s for s in out.reqs if id(s) not in did), key=lambda s: -s.num_new):
                j = min(range(n), key=lambda b: load[b])
                bins[j].append(s)
                load[j] += s.num_new
            return [SchedulerOutput(reqs=b) for b in bins if b]
        total = out.num_tokens
        mbs, cur, acc = [], [], 0
        for s in out.reqs:
            cur.append(s)
            acc += s.num_new
            if len(mbs) < n - 1 and acc >= total * (len(mbs) + 1) / n:
                mbs.append(SchedulerOutput(reqs=cur))
                cur = []
        if cur:
            mbs.append(SchedulerOutput(reqs=cur))
        return mbs

    def _execute_pp(self, out: SchedulerOutput) -> dict[str, list[int]]:
        """One step of this rank's pipeline stage (eager).  The boundary tensors of a micro-batch
        (hidden and residual) travel as one packed [2, T, H] buffer over NCCL p2p in the stage's TP
        column (the reference's packed hop, vllm_sm80/worker/pp_hop.py:52); sends are asynchronous so
        a stage computes its next micro-batch while the previous one is in flight.  Every rank runs
        the same scheduler, so shapes need no metadata message.  The last stage samples and
        broadcasts the tokens over the column."""
        import torch.distributed as dist

        st = self.st
        m = self.model
        H = self.mcfg.hidden_size
        hc = bool(self.mcfg.hc_mult)
        grp = st.pp_group
        sends, toks, nbytes = [], [], 0
        ev = self._ev_start()
        verify = {}
        mb_ctx = []
        mbs = self._micro_batches(out)
        out = SchedulerOutput(reqs=[s for mb in mbs for s in mb.reqs], preempted=out.preempted)
        for mb in mbs:
            h = self._host_inputs(mb)
            dev, ctx, nb = self._context(h)
            if self._spec_enabled_elsewhere():
                self._kda_verify_flags(mb, ctx)
                mb_ctx.append((mb, ctx))
            nbytes += nb
            if m.first:
                self._apply_pp_drafts(mb, dev["ids"])
                res = m(dev["ids"], ctx)
            elif hc:
                # hyper-connection streams: the whole mHC state as one packed uint8 message
                buf = torch.empty(hybrid.hc_hop_bytes(self.mcfg, h["T"]), dtype=torch.uint8, device=self.device)
                dist.recv(buf, src=st.pp_peer(st.pp_rank - 1), group=grp)
                res = m(None, ctx, hybrid.hc_unpack(buf, self.mcfg, h["T"]))
            else:
                # hidden, residual and the auxiliary hidden states of earlier stages' drafter layers
                n_aux = sum(1 for i in m.aux_layer_ids if i < m.layer_start)
                buf = torch.empty(2 + n_aux, h["T"], H, dtype=torch.bfloat16, device=self.device)
                dist.recv(buf, src=st.pp_peer(st.pp_rank - 1), group=grp)
                res = m(None, ctx, (buf[0], buf[1]))
                if m.aux_layer_ids:
                    m.aux_hidden = list(buf[2:]) + m.aux_hidden
            if not m.last:
                packed = hybrid.hc_pack(res, self.mcfg) if hc else torch.stack(list(res) + list(m.aux_hidden))
                sends.append((dist.isend(packed, dst=st.pp_peer(st.pp_rank + 1), group=grp), packed))
            elif self.spec is not None:
                rows = self._to_dev(h["sample_rows"])
                verify.update(self._verify_mb(mb, res, rows))
                # the drafter catches up over every position (MTP: final hidden; DFlash: aux states)
                self._pp_hidden.append((mb, res, list(m.aux_hidden)))
            else:
                rows = self._to_dev(h["sample_rows"])
                toks.append(self._sample_hidden(res, rows, self._sample_temps(mb, h), self.cfg.seed,
                                                self._sample_bans(mb)))
        for w, _ in sends:
            w.wait()
        if self._pp_drafts is not None:  # taken by this step; the other stages retire the broadcast here
            self._pp_drafts[2].wait()
            self._pp_drafts = None
        self.step_counter += 1
        last = st.pp_peer(st.pp_size - 1)
        if self._spec_enabled_elsewhere():
            res = self._pp_broadcast_lists(out, verify if m.last else None, self.cfg.scheduler.num_speculative_tokens + 1)
            self._pp_last_out, self._pp_last_res = out, res
            for mb, ctx in mb_ctx:
                self._kda_recover(mb, ctx, res)
        else:
            n = sum(1 for s in out.reqs if s.sample)
            tokens = torch.cat(toks) if m.last and toks else torch.empty(n, dtype=torch.int64, device=self.device)
            if n:
                dist.broadcast(tokens, src=last, group=grp)
            res = self._split_tokens(out, sanitize(tokens.cpu().tolist(), self.mcfg.vocab_size))
        self._ev_end(ev)
        self.last_stats = StepStats(num_tokens=out.num_tokens, graph=False, h2d_bytes=nbytes,
                                    d2h_bytes=8 * sum(len(v) for v in res.values()))
        if self._events is not None:
            self.last_stats.device_ms = self._events[0].elapsed_time(self._events[1])
            self._events = None
        if self.device.type == "cuda":
            _ext.check_status(self.device)
        return res

    def _pp_broadcast_lists(self, out: SchedulerOutput, lists: dict | None, width: int,
                            src_stage: int = -1) -> dict[str, list[int]]:
        """Token lists per request (accepted tokens of a verify step, or drafts) from the last pipeline
        stage (or ``src_stage``) to every stage of this TP column, as one int64 device tensor
        [requests, 1 + width] (count, tokens) in the step's request order, which every rank's scheduler
        shares: no pickled objects."""
        import torch.distributed as dist

        st = self.st
        rids = [s.req.request_id for s in out.reqs]
        buf = torch.full((len(rids), 1 + width), -1, dtype=torch.int64)
        if lists is not None:
            for i, rid in enumerate(rids):
                v = lists.get(rid)
                if v is not None:
                    buf[i, 0] = len(v)
                    buf[i, 1:1 + len(v)] = torch.tensor(v[:width], dtype=torch.int64)
        dev = buf.to(self.device) if self.device.type == "cuda" else buf
        src = st.pp_size - 1 if src_stage < 0 else src_stage
        dist.broadcast(dev, src=st.pp_peer(src), group=st.pp_group if self.device.type == "cuda" else st.pp_cpu_group)
        host = dev.cpu().tolist()
        return {rid: row[1:1 + row[0]] for rid, row in zip(rids, host) if row[0] >= 0}

    def _kda_verify_flags(self, out: SchedulerOutput, ctx) -> None:
        """Sequences verifying drafts through KDA layers record their updates instead of committing
        them (the state must end at the last accepted token)."""
        if not self.model.kda_layer_ids() or not any(s.num_draft for s in out.reqs):
            return
        flags = np.asarray([1 if s.num_draft else 0 for s in out.reqs], dtype=np.int32)
        ctx.kda_verify = self._to_dev(flags)

    def _kda_recover(self, out: SchedulerOutput, ctx, res: dict) -> None:
        if ctx.kda_verify is None:
            return
        keep = np.asarray([len(res.get(s.req.request_id, [])) if s.num_draft else 0 for s in out.reqs],
                          dtype=np.int32)
        keep = np.maximum(keep, np.asarray([1 if s.num_draft else 0 for s in out.reqs], dtype=np.int32))
        self.model.kda_recover(ctx, torch.from_numpy(keep))

    def _spec_enabled_elsewhere(self) -> bool:
        return self.cfg.scheduler.num_speculative_tokens > 0

    def _verify_mb(self, mb: SchedulerOutput, hidden, rows) -> dict[str, list[int]]:
        rows_of, k = {}, 0
        for s in mb.reqs:
            if s.sample:
                n = s.num_new if s.num_draft else 1
                rows_of[s.req.request_id] = list(range(k, k + n))
                k += n
        if not k:
            return {}
        logits = self.model.compute_logits(hidden.index_select(0, rows))
        return sanitize_dict(self.spec.verify(mb, logits, rows_of), self.mcfg.vocab_size)

    def _execute_spec(self, out: SchedulerOutput) -> dict[str, list[int]]:
        """Target step with draft verification (a captured graph per batch size and draft count when the
        step is uniform, else eager); the hidden states are kept for :meth:`propose`."""
        k = self._spec_graph_k(out)
        if k:
            return self._execute_spec_graph(out, k)
        h = self._host_inputs(out)
        dev, ctx, nbytes = self._context(h)
        self._kda_verify_flags(out, ctx)
        ev = self._ev_start()
        hidden = self.model(dev["ids"], ctx)
        rows_of = {}
        k = 0
        t = 0
        for s in out.reqs:
            if s.sample:
                n = s.num_new if s.num_draft else 1
                rows_of[s.req.request_id] = list(range(k, k + n))
                k += n
            t += s.num_new
        res = {}
        if k:
            logits = self.model.compute_logits(hidden.index_select(0, self._to_dev(h["sample_rows"])))
            res = sanitize_dict(self.spec.verify(out, logits, rows_of), self.mcfg.vocab_size)
        self._kda_recover(out, ctx, res)
        self._ev_end(ev)
        self.step_counter += 1
        stats = StepStats(num_tokens=out.num_tokens, graph=False, h2d_bytes=nbytes,
                          d2h_bytes=8 * sum(len(v) for v in res.values()))
        if self._events is not None:
            stats.device_ms = self._events[0].elapsed_time(self._events[1])
            self._events = None
        self.last_stats = stats
        self._pending = (out, hidden, res)
        if self.device.type == "cuda":
            _ext.check_status(self.device)
        return res

    @torch.inference_mode()
    def propose(self) -> None:
        """Draft tokens for the next step (speculative decoding; after the scheduler update).  With
        pipeline parallelism the last stage drafts and broadcasts the drafts to the other stages."""
        if self.cfg.scheduler.num_speculative_tokens <= 0:
            return
        if self.st.pp_size > 1:
            import torch.distributed as dist

            drafts = None
            if self._pp_last_out is not None and self._tail_step(self._pp_last_out):
                return self._propose_tail()
            if self.spec is not None:
                for mb, hidden, aux in self._pp_hidden:
                    self.model.aux_hidden = aux
                    self.spec.propose(mb, hidden, self._pp_accepted(mb))
                drafts = {s.req.request_id: list(s.req.draft_token_ids) for mb, _, _ in self._pp_hidden
                          for s in mb.reqs}
            self._pp_hidden = []
            if self._pp_last_out is None:
                return
            if self._split_drafts_on():
                self._pp_drafts_async(self._pp_last_out, drafts)
                return
            got = self._pp_broadcast_lists(self._pp_last_out, drafts, self.cfg.scheduler.num_speculative_tokens)
            if self.spec is None:
                for s in self._pp_last_out.reqs:
                    d = got.get(s.req.request_id)
                    if d is not None and not s.req.status.finished:
                        s.req.draft_token_ids = list(d)
            return
        if self.spec is None or self._pending is None:
            return
        out, hidden, res = self._pending
        self._pending = None
        self.spec.propose(out, hidden, res)

    _pp_last_out = None
    _pp_last_res: dict = {}
    _pp_drafts = None  # split draft event: (request -> row, the broadcast int64 [requests, 1 + k], its work)
    split_draft_events = 0  # asynchronous draft broadcasts this process issued (all runners)

    def _split_drafts_on(self) -> bool:
        """Split draft event (the reference's VLLM_PP_SPLIT_DRAFT_EVENT, vllm_sm80/worker/pp_handler.py:7-10,
        applied in runner_hooks.py:148-160): usable when every stage can name each request's draft count
        without the drafts (no verify-depth cut that depends on device features, no n-gram tables hashed
        from the tokens on the host)."""
        from .. import envs

        pol = getattr(self.spec, "depth", None) if self.spec is not None else None
        masked = self.cfg.scheduler.depth_mode == "mask" or (pol is None and not self.cfg.scheduler.depth_policy
                                                            and not envs.get("VLLM_B200_ADAPTIVE_DEPTH"))
        return bool(envs.get("VLLM_B200_PP_SPLIT_DRAFTS")) and masked and not self._ngram_sources()

    # ------------------------------------------------------------------ pipeline draft tail
    _tail_head = None  # tail stage: the lm_head shard received from the last stage
    _tail_sent = False  # last stage: the lm_head shard went to the tail stage
    draft_tail_steps = 0  # steps whose drafts a tail stage picked (all runners of this process)

    def _tail_stage(self) -> int:
        """The stage computing the DFlash drafter's tail (the reference's VLLM_PP_DRAFT_TAIL_STAGE,
        vllm_sm80/worker/pp_handler.py:11-14 and worker/pp_draft_tail.py), or -1.  The block drafter's
        forward stays beside the target's last layers (it reads their auxiliary states); the tail --
        the lm_head over k rows per request and the picks -- moves to a stage that is otherwise idle
        while the last stage finishes, which roots the drafts' broadcast."""
        from .. import envs

        v = int(envs.get("VLLM_B200_PP_DRAFT_TAIL_STAGE"))
        sch = self.cfg.scheduler
        if (v < 0 or v >= self.st.pp_size - 1 or sch.spec_method != "dflash" or sch.depth_policy
                or envs.get("VLLM_B200_ADAPTIVE_DEPTH") or self._ngram_sources()):
            return -1
        return v

    def _tail_reqs(self, out: SchedulerOutput) -> list:
        """The requests that keep decoding after the step (the drafter's rule, on every stage)."""
        return [s.req for s in out.reqs if not s.req.status.finished
                and s.req.num_computed_tokens == s.req.num_tokens - 1]

    def _tail_step(self, out: SchedulerOutput) -> bool:
        """The tail moves this step: a tail stage is set and every drafting request picks greedily (a
        sampled draft's probabilities must stay beside the verifier on the last stage)."""
        return self._tail_stage() >= 0 and all(q.params.temperature <= 0 for q in self._tail_reqs(out))

    def _propose_tail(self) -> None:
        """Last stage: the block forward per micro-batch, its hidden states [A, k, H] to the tail stage
        (with the lm_head shard once, the first time).  Tail stage: the logits and greedy picks, then the
        drafts' broadcast from there; every stage stores the drafts it receives."""
        import torch.distributed as dist

        st = self.st
        out = self._pp_last_out
        tail = self._tail_stage()
        k = self.cfg.scheduler.num_speculative_tokens
        grp = st.pp_group
        areqs = self._tail_reqs(out)
        H = self.mcfg.hidden_size
        drafts = None
        if self.spec is not None:  # last stage
            parts = []
            for mb, hidden, aux in self._pp_hidden:
                self.model.aux_hidden = aux
                got = self.spec.propose(mb, hidden, self._pp_accepted(mb), defer_tail=True)
                if got is not None:
                    parts.append(got[1])
            self._pp_hidden = []
            if not self._tail_sent:
                dist.send(self.model.lm_head.weight.data.contiguous(), dst=st.pp_peer(tail), group=grp)
                self._tail_sent = True
            if areqs:
                h = torch.cat(parts).contiguous()
                assert h.shape == (len(areqs), k, H), "the drafter's requests differ from the stage's rule"
                dist.send(h, dst=st.pp_peer(tail), group=grp)
        elif st.pp_rank == tail:
            if self._tail_head is None:
                w = torch.empty(self.model.vocab_local, H, dtype=torch.bfloat16, device=self.device)
                dist.recv(w, src=st.pp_peer(st.pp_size - 1), group=grp)
                from ..models.layers import Linear

                self._tail_head = Linear(w)
            if areqs:
                from .spec_decode import _SEED_DRAFT, _sample

                h = torch.empty(len(areqs), k, H, dtype=torch.bfloat16, device=self.device)
                dist.recv(h, src=st.pp_peer(st.pp_size - 1), group=grp)
                picks = [_sample(self._tail_head(h[:, j].contiguous()), None, self.cfg.seed ^ (_SEED_DRAFT + j),
                                 self.step_counter, self.model.vocab_offset) for j in range(k)]
                dh = torch.stack(picks, dim=1).cpu().tolist()
                drafts = {}
                for a, req in enumerate(areqs):
                    room = max(0, req.params.max_tokens - len(req.output_token_ids) - 1)
                    drafts[req.request_id] = [int(v) for v in dh[a][:max(0, min(k, room))]]
        got = self._pp_broadcast_lists(out, drafts, k, src_stage=tail)
        ModelRunner.draft_tail_steps += 1
        for req in areqs:
            req.draft_token_ids = list(got.get(req.request_id, []))
            req.draft_live = -1

    def _pp_drafts_async(self, out: SchedulerOutput, drafts: dict | None) -> None:
        """Send the last stage's drafts over the stage column without waiting; the other stages set each
        continuing request's draft count now (placeholder ids) and the first stage takes the ids from the
        broadcast right before its next forward."""
        import torch.distributed as dist

        st = self.st
        k = self.cfg.scheduler.num_speculative_tokens
        rids = [s.req.request_id for s in out.reqs]
        buf = torch.full((len(rids), 1 + k), -1, dtype=torch.int64)
        if drafts is not None:
            for i, rid in enumerate(rids):
                v = drafts.get(rid)
                if v is not None:
                    buf[i, 0] = len(v)
                    buf[i, 1:1 + len(v)] = torch.tensor(v[:k], dtype=torch.int64)
        dev = buf.to(self.device) if self.device.type == "cuda" else buf
        work = dist.broadcast(dev, src=st.pp_peer(st.pp_size - 1), group=st.pp_group if self.device.type == "cuda"
                              else st.pp_cpu_group, async_op=True)
        self._pp_drafts = ({rid: i for i, rid in enumerate(rids)}, dev, work)
        ModelRunner.split_draft_events += 1
        if self.spec is None:
            for s in out.reqs:
                req = s.req
                # the drafter's own count rule: requests that keep decoding draft min(k, room) tokens
                if req.status.finished or req.num_computed_tokens != req.num_tokens - 1:
                    continue
                room = max(0, req.params.max_tokens - len(req.output_token_ids) - 1)
                req.draft_token_ids = [-1] * max(0, min(k, room))

    def _apply_pp_drafts(self, mb: SchedulerOutput, ids: torch.Tensor) -> None:
        """First stage, split draft event: wait for the drafts' broadcast on the stream (as late as
        possible) and put the ids into this micro-batch's input rows."""
        if self._pp_drafts is None:
            return
        row_of, buf, work = self._pp_drafts
        work.wait()
        dst, src = [], []
        t = 0
        w = buf.shape[1]
        for s in mb.reqs:
            r = row_of.get(s.req.request_id)
            if s.num_draft and r is not None:
                for j in range(s.num_draft):  # drafts follow the request's first token of the step
                    dst.append(t + 1 + j)
                    src.append(r * w + 1 + j)
            t += s.num_new
        if dst:
            ids[self._to_dev(np.asarray(dst, dtype=np.int64))] = buf.view(-1)[self._to_dev(np.asarray(src, dtype=np.int64))]

    def _pp_accepted(self, mb) -> dict:
        return {s.req.request_id: self._pp_last_res.get(s.req.request_id, []) for s in mb.reqs}

    def _ev_start(self):
        if not (self.time_device and self.device.type == "cuda"):
            return None
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        return (a, b)

    def _ev_end(self, ev):
        if ev is not None:
            ev[1].record()
            self._events = ev

    def _sample_bans(self, out):
        """[sampled rows, MAX_BANS] banned token ids on the device, or None when no request bans any."""
        if not any(s.req.params.bad_token_ids for s in out.reqs if s.sample):
            return None
        rows = [s for s in out.reqs if s.sample]
        assert all(s.num_draft == 0 for s in rows), "banned tokens with speculative decoding"
        return self._to_dev(self._bans_rows(rows, len(rows)))

    def _sample_temps(self, out, h):
        temps = []
        for s in out.reqs:
            if s.sample:
                temps.extend([s.req.params.temperature] * (s.num_new if s.num_draft else 1))
        if not temps or all(t <= 0 for t in temps):
            return None
        return self._to_dev(np.asarray(temps, dtype=np.float32))

    @staticmethod
    def _split_tokens(out: SchedulerOutput, host: list[int]) -> dict[str, list[int]]:
        res = {}
        k = 0
        for s in out.reqs:
            if not s.sample:
                continue
            if s.num_draft:
                # verify: accept drafts while they match the target's choice, then the bonus token
                cand = host[k:k + s.num_new]
                k += s.num_new
                live = s.num_draft if s.req.draft_live < 0 else min(s.num_draft, s.req.draft_live)
                drafts = s.req.draft_token_ids[:live]
                acc = []
                for j, d in enumerate(drafts):
                    acc.append(cand[j])
                    if cand[j] != d:
                        break
                else:
                    acc.append(cand[live])
                res[s.req.request_id] = acc
            else:
                res[s.req.request_id] = [host[k]]
                k += 1
        return res

    # ------------------------------------------------------------------ CUDA graphs
    def _capture(self, B: int):
        dev = self.device
        mml = self.cfg.scheduler.max_model_len
        # the per-step inputs are views of one device buffer, filled by one copy from one pinned
        # host buffer of the same layout (fields 16-byte aligned)
        specs = [("ids", (B,), torch.int64), ("pos", (B,), torch.int32), ("slots", (B,), torch.int64),
                 ("tseq", (B,), torch.int32), ("ctx", (B,), torch.int32), ("cu", (B + 1,), torch.int32),
                 ("kslot", (B,), torch.int32), ("hinit", (B,), torch.int32),
                 ("bt", (B, self.max_blocks_per_seq), torch.int32), ("temps", (B,), torch.float32),
                 ("bans", (B, sampling_ops.MAX_BANS), torch.int32)]
        for name, src in self._ngram_sources():
            specs.append((name, (B, src.heads), torch.int64))
        bufs, host, devbuf, hviews = self._graph_buffers(specs)
        bufs["slots"].fill_(-1)
        bufs["tseq"].copy_(torch.arange(B, dtype=torch.int32))
        bufs["ctx"].fill_(1)
        bufs["cu"].copy_(torch.arange(B + 1, dtype=torch.int32))
        bufs["bans"].fill_(-1)
        bufs["scores"] = torch.empty(B, mml, dtype=torch.float32, device=dev)
        ctx = StepContext(positions=bufs["pos"], num_tokens=B, slot_mapping=bufs["slots"], token_seq=bufs["tseq"],
                          ctx_lens=bufs["ctx"], block_table=bufs["bt"], max_ctx=mml, cu_seqlens=bufs["cu"],
                          kda_slots=bufs["kslot"], has_init=bufs["hinit"], mla_caches=self.mla_caches,
                          kda_states=self.kda_states, scores_buf=bufs["scores"], dsa_cores=self.dsa_cores,
                          gqa_caches=self.gqa_caches, ple_ids=bufs.get("ple"),
                          engram_ids=bufs.get("engram"))
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self._forward_sample(bufs["ids"], ctx, None, bufs["temps"], self.cfg.seed, bufs["bans"])
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        if self.graph_pool is None:
            self.graph_pool = torch.cuda.graph_pool_handle()
        with torch.cuda.graph(g, pool=self.graph_pool):
            ids_out = self._forward_sample(bufs["ids"], ctx, None, bufs["temps"], self.cfg.seed, bufs["bans"])
        torch.cuda.synchronize(dev)
        self.graphs[B] = (g, bufs, ids_out)
        self._packed[B] = (host, devbuf, hviews)

    def _graph_buffers(self, specs):
        """Device views of one buffer for a graph's per-step inputs, filled by one copy from a pinned host
        buffer of the same layout (fields 16-byte aligned): (device views, host, device, host views)."""
        offs, off = {}, 0
        for k, shape, dt in specs:
            offs[k] = off
            off += (math.prod(shape) * torch.empty((), dtype=dt).element_size() + 15) // 16 * 16
        host = torch.zeros(off, dtype=torch.uint8, pin_memory=True)
        devbuf = torch.zeros(off, dtype=torch.uint8, device=self.device)
        bufs, hviews = {}, {}
        for k, shape, dt in specs:
            nb = math.prod(shape) * torch.empty((), dtype=dt).element_size()
            bufs[k] = devbuf[offs[k]:offs[k] + nb].view(dt).view(shape)
            hviews[k] = host[offs[k]:offs[k] + nb].view(dt).view(shape).numpy()
        return bufs, host, devbuf, hviews

    # ------------------------------------------------------------------ speculative verify graphs
    def _spec_graph_k(self, out: SchedulerOutput) -> int:
        """The draft count k when this verify step replays a captured graph (one graph per batch size
        and draft count, the reference's adaptive-k graphs, vllm_sm80/worker/adaptive_k_graphs.py:35-119):
        every request verifies exactly k drafts from a non-empty context, one pipeline stage, graphs on.
        0 otherwise (the eager path)."""
        if (self.cfg.enforce_eager or not self.graphs_ok or self.device.type != "cuda" or self.st.pp_size > 1
                or self.dsa_cores or not out.reqs or len(out.reqs) > max(self.cfg.cuda_graph_batch_sizes)):
            return 0
        k = out.reqs[0].num_draft
        if k <= 0 or any(s.num_draft != k or s.num_new != k + 1 or not s.sample or s.start == 0 for s in out.reqs):
            return 0
        return k

    def _host_inputs_spec(self, out: SchedulerOutput, Bp: int, k: int) -> dict:
        """Inputs of a uniform verify step padded to Bp sequences of k + 1 tokens (padding: no cache rows
        written, KDA updates only recorded)."""
        reqs = out.reqs
        n = k + 1
        T = Bp * n
        ids = np.zeros(T, dtype=np.int64)
        pos = np.tile(np.arange(n, dtype=np.int32), Bp)
        slots = np.full(T, -1, dtype=np.int64)
        ctx = pos + 1
        kslot = np.zeros(Bp, dtype=np.int32)
        hinit = np.zeros(Bp, dtype=np.int32)
        bt = np.zeros((Bp, self.max_blocks_per_seq), dtype=np.int32)
        for i, s in enumerate(reqs):
            r = s.req
            a = s.start
            ids[i * n:(i + 1) * n] = r.tokens(a, a + 1) + list(r.draft_token_ids[:k])
            p = np.arange(a, a + n, dtype=np.int64)
            pos[i * n:(i + 1) * n] = p
            ctx[i * n:(i + 1) * n] = p + 1
            b = np.asarray(r.block_ids, dtype=np.int64)
            slots[i * n:(i + 1) * n] = b[p // 64] * 64 + p % 64
            kslot[i] = max(r.kda_slot, 0)
            hinit[i] = 1
            bt[i] = self._bt_row(r)
        h = dict(ids=ids, pos=pos, slots=slots, ctx=ctx, kslot=kslot, hinit=hinit, bt=bt)
        self._add_ngram_ids(h, ((s.req, s.start, n, k) for s in reqs), Bp * n)
        return h

    def _capture_spec(self, Bp: int, k: int) -> None:
        dev = self.device
        mml = self.cfg.scheduler.max_model_len
        n = k + 1
        T = Bp * n
        specs = [("ids", (T,), torch.int64), ("pos", (T,), torch.int32), ("slots", (T,), torch.int64),
                 ("ctx", (T,), torch.int32), ("kslot", (Bp,), torch.int32), ("hinit", (Bp,), torch.int32),
                 ("bt", (Bp, self.max_blocks_per_seq), torch.int32)]
        for name, src in self._ngram_sources():
            specs.append((name, (T, src.heads), torch.int64))
        bufs, host, devbuf, hviews = self._graph_buffers(specs)
        bufs["slots"].fill_(-1)
        bufs["ctx"].fill_(1)
        bufs["tseq"] = torch.arange(Bp, dtype=torch.int32, device=dev).repeat_interleave(n)
        bufs["cu"] = torch.arange(0, T + 1, n, dtype=torch.int32, device=dev)
        bufs["scores"] = torch.empty(T, mml, dtype=torch.float32, device=dev)
        verify = torch.ones(Bp, dtype=torch.int32, device=dev) if self.model.kda_layer_ids() else None
        ctx = StepContext(positions=bufs["pos"], num_tokens=T, slot_mapping=bufs["slots"], token_seq=bufs["tseq"],
                          ctx_lens=bufs["ctx"], block_table=bufs["bt"], max_ctx=mml, cu_seqlens=bufs["cu"],
                          kda_slots=bufs["kslot"], has_init=bufs["hinit"], mla_caches=self.mla_caches,
                          kda_states=self.kda_states, scores_buf=bufs["scores"], dsa_cores=self.dsa_cores,
                          gqa_caches=self.gqa_caches, ple_ids=bufs.get("ple"),
                          engram_ids=bufs.get("engram"), kda_verify=verify)

        def fwd():
            hidden = self.model(bufs["ids"], ctx)
            return hidden, self.model.compute_logits(hidden)

        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                fwd()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        if self.graph_pool is None:
            self.graph_pool = torch.cuda.graph_pool_handle()
        with torch.cuda.graph(g, pool=self.graph_pool):
            hidden, logits = fwd()
        torch.cuda.synchronize(dev)
        self.spec_graphs[(Bp, k)] = (g, bufs, ctx, hidden, logits, list(self.model.aux_hidden or []),
                                     (host, devbuf, hviews))

    def _execute_spec_graph(self, out: SchedulerOutput, k: int) -> dict[str, list[int]]:
        Bp = next(b for b in sorted(self.cfg.cuda_graph_batch_sizes) if b >= len(out.reqs))
        if (Bp, k) not in self.spec_graphs:
            self._capture_spec(Bp, k)
        g, bufs, ctx, hidden_all, logits_all, aux, (host, devbuf, hviews) = self.spec_graphs[(Bp, k)]
        h = self._host_inputs_spec(out, Bp, k)
        for name, v in hviews.items():
            np.copyto(v, h[name])
        devbuf.copy_(host, non_blocking=True)
        ev = self._ev_start()
        g.replay()
        n, S = k + 1, len(out.reqs)
        rows_of = {s.req.request_id: list(range(i * n, (i + 1) * n)) for i, s in enumerate(out.reqs)}
        res = sanitize_dict(self.spec.verify(out, logits_all[:S * n], rows_of), self.mcfg.vocab_size)
        if ctx.kda_verify is not None:
            keep = np.zeros(Bp, dtype=np.int32)
            keep[:S] = [max(1, len(res.get(s.req.request_id, []))) for s in out.reqs]
            self.model.kda_recover(ctx, torch.from_numpy(keep))
        self._ev_end(ev)
        self.step_counter += 1
        stats = StepStats(num_tokens=out.num_tokens, graph=True, h2d_bytes=host.numel(),
                          d2h_bytes=8 * sum(len(v) for v in res.values()))
        if self._events is not None:
            stats.device_ms = self._events[0].elapsed_time(self._events[1])
            self._events = None
        self.last_stats = stats
        self.model.aux_hidden = list(aux)
        self._pending = (out, hidden_all[:S * n], res)
        _ext.check_status(self.device)
        return res

    def _stage_graph_inputs(self, B: int, h: dict) -> int:
        """Write the step's inputs into the graph's pinned host buffer and copy it to the device in one
        transfer (the previous step's copy has completed: every step reads its tokens back)."""
        host, devbuf, hviews = self._packed[B]
        for k, v in hviews.items():
            np.copyto(v, h[k])
        devbuf.copy_(host, non_blocking=True)
        return host.numel()

    def capture_graphs(self) -> dict[int, int]:
        """Capture the decode graph of every configured batch size up front and return the device
        bytes each capture kept (growth of the allocator's reserved memory across the capture; the
        graphs share one pool, so later sizes reuse what earlier ones reserved).  The reference
        measures the same quantity to split its graph-memory budget
        (vllm_sm80/worker/cudagraph_mem.py:202-284)."""
        kept = {}
        self.graph_transient = {}
        if self.device.type != "cuda" or self.cfg.enforce_eager or self.st.pp_size > 1 or not self.graphs_ok:
            return kept
        for B in sorted(self.cfg.cuda_graph_batch_sizes):
            if B in self.graphs or B > self.cfg.scheduler.max_num_seqs:
                continue
            torch.cuda.synchronize(self.device)
            before = torch.cuda.memory_reserved(self.device)
            torch.cuda.reset_peak_memory_stats(self.device)
            self._capture(B)
            torch.cuda.synchronize(self.device)
            kept[B] = torch.cuda.memory_reserved(self.device) - before
            # transient: what the capture (its eager warm-up runs included) allocated at its peak and freed
            # again -- needed free while capturing, not kept afterwards (the reference splits the same two,
            # vllm_sm80/worker/cudagraph_mem.py:202-284)
            self.graph_transient[B] = max(0, torch.cuda.max_memory_allocated(self.device)
                                          - torch.cuda.memory_allocated(self.device))
        return kept

    graph_transient: dict = {}

    @torch.inference_mode()
    def warmup(self) -> None:
        """Run one prefill and one decode step of a throwaway request through every kernel family
        the model uses, before any graph is captured or request served: per-kernel attributes, the
        status word and cached work items are set up outside capture (the reference's kernel
        warm-up driver, vllm_sm80/kernels/warmup.py:38)."""
        from .request import Request, SamplingParams
        from .scheduler import ScheduledReq

        n = max(2, min(64, self.cfg.scheduler.max_model_len // 2))
        req = Request(list(range(1, n + 1)), SamplingParams(max_tokens=2), request_id="__warmup__")
        need = (n + 2 + self.block_size - 1) // self.block_size
        if self.block_pool.num_free() < need:
            return
        req.block_ids = [int(b) for b in self.block_pool.allocate(need)]
        if self.slot_pool is not None:
            req.kda_slot = self.slot_pool.allocate()
        try:
            saved = self.cfg.enforce_eager
            self.cfg.enforce_eager = True
            try:
                self.execute(SchedulerOutput(reqs=[ScheduledReq(req, n, 0, True)]))
                req.output_token_ids.append(1)
                req.num_computed_tokens = n
                self.execute(SchedulerOutput(reqs=[ScheduledReq(req, 1, n, True)]))
            finally:
                self.cfg.enforce_eager = saved
        finally:
            self.block_pool.free(req.block_ids)
            if self.slot_pool is not None and req.kda_slot > 0:
                self.slot_pool.free(req.kda_slot)
            self._pending = None
            if self.spec is not None:
                self.spec.q_store.clear()
            if self.device.type == "cuda":
                torch.cuda.synchronize(self.device)

    def release_graphs(self):
        self.graphs.clear()
        self._packed.clear()
        self.spec_graphs.clear()
        self.graph_pool = None
