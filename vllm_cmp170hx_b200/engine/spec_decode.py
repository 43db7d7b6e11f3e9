"""Speculative decoding with an MTP draft head: verification, rejection
sampling and proposal over vocab-sharded logits.

A request verified with k drafts d_1..d_k computes positions p..p+k holding
[last, d_1..d_k]; the target's logits row j scores the token after position
p+j.  Greedy requests accept drafts while they equal the target's argmax and
take the target's token at the first mismatch (the bonus token after k
accepts).  Sampled requests use speculative rejection sampling: accept d_j
with probability min(1, p_j(d_j) / q_j(d_j)); at the first rejection sample
from normalize(max(0, p_j - q_j)); after k accepts sample the bonus from
p_k, where p is the target's tempered softmax and q the draft's.  The
resulting tokens are distributed exactly as the target's own samples.

Everything is batched over the step's rows and stays on the device until a
single host copy: with tensor parallel the vocab is sharded, maxima and sums
are all-reduced, the draft token's probability comes from its owning shard,
and residual/bonus draws are Gumbel-max per shard (the sampling kernel, whose
noise is indexed by global vocab id) combined across ranks, so logits are
never gathered (the reference shards its argmax the same way,
vllm_sm80/spec_decode/shard_argmax.py).  Acceptance uniforms come from a
host generator seeded by (seed, step), identical on every rank.

Proposal (the DeepSeek MTP drafter of the reference's config 5): after the
target step the MTP head catches up over the positions the target just
computed -- position i takes token i+1 and the target's final hidden h_i --
and then chains k-1 single-token steps on its own hidden state.  With the
DFlash block drafter (models/dflash.py) the step's verified positions are
stored as context rows from the target's auxiliary hidden states and all k
drafts come from one non-causal forward of [bonus, mask x k].  The drafts
of all requests are produced together and copied to the host once.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from .. import envs
from ..models.hybrid import StepContext
from ..ops import sampling as sampling_ops
from ..parallel import comm
from ..parallel import state as pstate
from .depth_policy import logit_stats

_SEED_VERIFY = 0x5BD1E995
_SEED_DRAFT = 0x27D4EB2F


def _live_drafts(req, num_draft: int) -> int:
    """Drafts of a verify step that are candidates (the row mask's live depth, at most the scheduled)."""
    return num_draft if req.draft_live < 0 else min(num_draft, req.draft_live)


def _all_reduce(x: torch.Tensor, op=dist.ReduceOp.SUM) -> torch.Tensor:
    st = pstate.get()
    if st.tp_size > 1 and not st.emulated:
        dist.all_reduce(x, op=op, group=st.tp_group)
    return x


def _sample(logits: torch.Tensor, temps: torch.Tensor | None, seed: int, step: torch.Tensor | None, off: int):
    """Token ids [rows] (device int64) of greedy/Gumbel sampling over the sharded vocab."""
    val, idx = sampling_ops.sample_local(logits, temps, seed, step, off)
    if pstate.get().tp_size > 1:
        return sampling_ops.combine(comm.tp_all_gather(val[None], 0), comm.tp_all_gather(idx[None], 0))
    return idx.long()


def tempered_probs(logits: torch.Tensor, temps: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(unnormalised exp(l/T - max) of this shard [rows, V_local], global sums [rows])."""
    z = logits.float() / temps[:, None]
    m = _all_reduce(z.max(dim=-1).values.contiguous(), dist.ReduceOp.MAX)
    e = torch.exp(z - m[:, None])
    return e, e.sum(-1)


class SpecDecoder:
    """MTP drafter + verifier bound to a :class:`ModelRunner`."""

    def __init__(self, runner, k: int):
        self.runner = runner
        self.k = k
        cfg = runner.cfg
        rows = runner.num_blocks * 64
        self.method = cfg.scheduler.spec_method
        init_mode = getattr(runner.model, "init_mode", "local")
        self.mtp = self.dflash = None
        if self.method == "dflash":
            from ..models.dflash import DFlashConfig, DFlashDrafter

            if cfg.model.hc_mult:
                raise NotImplementedError("the DFlash drafter reads plain residual streams (no hyper-connections)")
            dc = DFlashConfig(num_layers=cfg.scheduler.dflash_layers)
            self.dflash = DFlashDrafter(cfg.model, dc, runner.model, runner.device, cfg.seed, init_mode)
            runner.model.aux_layer_ids = tuple(self.dflash.dc.aux_layer_ids)
            self.dcaches = self.dflash.alloc_caches(rows, runner.device,
                                                    cfg.scheduler.max_num_seqs * (self.k + 1))
        elif self.method == "mtp":
            from ..models.mtp import MTPHead

            self.mtp = MTPHead(cfg.model, runner.model, runner.device, cfg.seed, init_mode)
            if self.mtp.kind == "gqa":
                runner.gqa_caches[self.mtp.layer_id] = torch.zeros(
                    *self.mtp.layer.attn.cache_rows(rows), dtype=torch.bfloat16, device=runner.device)
            else:
                runner.mla_caches[self.mtp.layer_id] = (
                    torch.zeros(rows, 576, dtype=torch.bfloat16, device=runner.device),
                    torch.zeros(rows, 128, dtype=torch.uint8, device=runner.device),
                    torch.ones(rows, dtype=torch.float32, device=runner.device))
        else:
            raise ValueError(f"unknown speculative method {self.method!r}")
        self.depth = None
        path = cfg.scheduler.depth_policy or envs.get("VLLM_B200_ADAPTIVE_DEPTH")
        if path:
            from .depth_policy import DepthPolicy

            self.depth = DepthPolicy.load(path)
            if self.depth.uses_conf and self.dflash is None:
                raise ValueError("the depth policy reads a confidence head, which only the DFlash drafter has")
        self.step_no = 0
        # draft distributions of sampled requests: rid -> (tensor [k, A, V_local], row a)
        self.q_store: dict[str, tuple[torch.Tensor, int]] = {}
        self.stats = {"proposed": 0, "accepted": 0, "steps": 0}
        self._last_p = None
        self.p_rounds: dict = {}  # request -> p_i rows of its latest drafted rounds (host width of the depth policy)

    # ------------------------------------------------------------------ verification
    def verify(self, out, logits: torch.Tensor, rows_of: dict[str, list[int]]) -> dict[str, list[int]]:
        """logits: this rank's shard [R, V_local] of the sampled rows; rows_of: request -> its rows, in order."""
        r = self.runner
        off = r.model.vocab_offset
        dev = logits.device
        self.step_no += 1
        greedy = _sample(logits, None, 0, None, off)
        # sampled requests: probabilities of the drafts and the residual / bonus draws
        trows, ttemps, tdraft, tq = [], [], [], []
        for s in out.reqs:
            req = s.req
            if not s.sample or req.params.temperature <= 0:
                continue
            rows = rows_of[req.request_id]
            qs = self.q_store.get(req.request_id)
            for j, row in enumerate(rows):
                trows.append(row)
                ttemps.append(req.params.temperature)
                d = req.draft_token_ids[j] if j < _live_drafts(req, s.num_draft) else -1
                tdraft.append(d)
                tq.append((qs, j) if (d >= 0 and qs is not None) else None)
        host_stats = None
        final = None
        if trows:
            sel = torch.tensor(trows, device=dev)
            temps = torch.tensor(ttemps, dtype=torch.float32, device=dev)
            e, ssum = tempered_probs(logits.index_select(0, sel), temps)
            Vl = e.shape[1]
            q = torch.zeros_like(e)
            for i, t in enumerate(tq):
                if t is not None:
                    qs, j = t
                    q[i] = qs[0][j, qs[1]]
            d = torch.tensor(tdraft, dtype=torch.int64, device=dev) - off
            own = (d >= 0) & (d < Vl)
            dl = d.clamp(0, Vl - 1)[:, None]
            pd = torch.where(own, e.gather(1, dl)[:, 0], 0.0)
            qd = torch.where(own, q.gather(1, dl)[:, 0], 0.0)
            st = _all_reduce(torch.stack([ssum, pd, qd], dim=1).contiguous())
            p = e / st[:, :1]
            resid = torch.clamp(p - q, min=0.0)  # bonus rows: q = 0 -> p
            ones = torch.ones(len(trows), dtype=torch.float32, device=dev)
            final = _sample(torch.log(resid), ones, r.cfg.seed ^ _SEED_VERIFY, r.step_counter, off)
            host_stats = st
        g_host = greedy.cpu().tolist()
        f_host = final.cpu().tolist() if final is not None else []
        if host_stats is not None:
            hs = host_stats.cpu().numpy()
            pd_h = hs[:, 1] / np.maximum(hs[:, 0], 1e-30)
            qd_h = hs[:, 2]
            gen = torch.Generator().manual_seed((r.cfg.seed * 1000003 + self.step_no) & 0x7FFFFFFFFFFF)
            u = torch.rand(len(trows), generator=gen, dtype=torch.float64).numpy()
        res = {}
        ti = 0
        for s in out.reqs:
            if not s.sample:
                continue
            req = s.req
            rows = rows_of[req.request_id]
            # masked draft rows (past the request's live depth) were verified but are not candidates:
            # the token at the first masked position is the target's own (greedy) or a draw from p
            drafts = req.draft_token_ids[: _live_drafts(req, s.num_draft)]
            acc = []
            if req.params.temperature <= 0:
                for j, dtok in enumerate(drafts):
                    acc.append(g_host[rows[j]])
                    if acc[-1] != dtok:
                        break
                else:
                    acc.append(g_host[rows[len(drafts)]])
            else:
                base = ti
                ti += len(rows)
                for j, dtok in enumerate(drafts):
                    qd = qd_h[base + j] if tq[base + j] is not None else 1.0
                    if qd > 0 and u[base + j] < min(1.0, pd_h[base + j] / qd):
                        acc.append(dtok)
                        continue
                    acc.append(f_host[base + j])
                    break
                else:
                    acc.append(f_host[base + len(drafts)])
            self.stats["proposed"] += len(drafts)
            self.stats["accepted"] += sum(1 for a, b in zip(acc, drafts) if a == b)
            res[req.request_id] = acc
        self.stats["steps"] += 1
        return res

    # ------------------------------------------------------------------ proposal
    def propose(self, out, hidden: torch.Tensor, accepted: dict[str, list[int]], defer_tail: bool = False):
        """Set ``draft_token_ids`` of the step's unfinished requests (call after the scheduler update).
        ``defer_tail`` (DFlash, pipeline draft tail): stop after the block forward and return the
        requests that keep decoding with the block's hidden states [A, k, H], whose logits and picks
        another stage computes."""
        r = self.runner
        dev = r.device
        for s in out.reqs:
            self.q_store.pop(s.req.request_id, None)
        if self.dflash is not None:
            return self._propose_dflash(out, accepted, defer_tail)
        ids, pos, hrows, tseq, reqs = [], [], [], [], []
        last = []
        t = 0
        for s in out.reqs:
            req = s.req
            n_rows = s.num_new
            base = t
            t += n_rows
            if s.num_draft:
                toks = accepted.get(req.request_id, [])
            else:
                toks = req.tokens(s.start + 1, min(s.start + s.num_new + 1, req.num_tokens))
            m = min(len(toks), n_rows)
            if m == 0:
                continue
            reqs.append(req)
            for j in range(m):
                ids.append(toks[j])
                pos.append(s.start + j)
                hrows.append(base + j)
                tseq.append(len(reqs) - 1)
            last.append(len(ids) - 1)
        if not ids:
            return
        ctx = self._ctx(pos, tseq, reqs)
        hs = hidden.index_select(0, torch.tensor(hrows, device=dev))
        x = self.mtp(torch.tensor(ids, device=dev), hs, ctx)
        # chain over the requests that keep decoding
        act = [i for i, req in enumerate(reqs)
               if not req.status.finished and req.num_computed_tokens == req.num_tokens - 1]
        if not act:
            return
        areqs = [reqs[i] for i in act]
        cur = x.index_select(0, torch.tensor([last[i] for i in act], device=dev))
        cur_pos = [pos[last[i]] for i in act]
        A = len(areqs)
        temps_l = [q.params.temperature for q in areqs]
        temps = torch.tensor(temps_l, dtype=torch.float32, device=dev) if any(v > 0 for v in temps_l) else None
        samp = [i for i, v in enumerate(temps_l) if v > 0]
        qbuf = torch.empty(self.k, len(samp), r.model.vocab_local, dtype=torch.float32, device=dev) if samp else None
        drafts, stats = [], []
        for j in range(self.k):
            logits = self.mtp.compute_logits(cur)
            tok = _sample(logits, temps, r.cfg.seed ^ (_SEED_DRAFT + j), r.step_counter, r.model.vocab_offset)
            if self.depth is not None and self.depth.uses_stats:
                stats.append(logit_stats(logits, _all_reduce))
            if samp:
                sel = torch.tensor(samp, device=dev)
                e, ssum = tempered_probs(logits.index_select(0, sel), temps.index_select(0, sel))
                qbuf[j] = e / ssum[:, None]
            drafts.append(tok)
            if j + 1 == self.k:
                break
            cur_pos = [p + 1 for p in cur_pos]
            ctx = self._ctx(cur_pos, list(range(A)), areqs)
            cur = self.mtp(tok, cur, ctx)
        live = self._live(A, stats, None)
        dh = torch.stack(drafts, dim=1).cpu().tolist()
        self._set_drafts(areqs, dh, live)
        for qi, a in enumerate(samp):
            self.q_store[areqs[a].request_id] = (qbuf, qi)

    def p_round(self, request_id: str, lag: int):
        """The p_i row of the request's verify round ``lag`` rounds before the one being scheduled
        (whose drafts were the latest drafted), or None."""
        rows = self.p_rounds.get(request_id)
        return rows[-1 - lag] if rows is not None and len(rows) > lag else None

    def _set_drafts(self, areqs, dh, live) -> None:
        """Store each request's drafts: cut to its live depth, or (depth_mode "mask") all k with the live
        depth recorded as the row mask."""
        if self._last_p is not None:
            from collections import deque

            keep = self.depth.host_width.lag + 1
            for a, req in enumerate(areqs):
                self.p_rounds.setdefault(req.request_id, deque(maxlen=keep)).append(self._last_p[a])
            self._last_p = None
        mask = self.runner.cfg.scheduler.depth_mode == "mask" and self.depth is not None
        for a, req in enumerate(areqs):
            room = max(0, req.params.max_tokens - len(req.output_token_ids) - 1)
            if mask:
                req.draft_token_ids = [int(v) for v in dh[a][:min(self.k, room)]]
                req.draft_live = max(0, min(live[a], len(req.draft_token_ids)))
            else:
                req.draft_token_ids = [int(v) for v in dh[a][:max(0, min(self.k, live[a], room))]]
                req.draft_live = -1

    def _live(self, A: int, stats: list, conf) -> list[int]:
        """Drafts worth verifying per request (all k without a depth policy)."""
        if self.depth is None:
            return [self.k] * A
        from .depth_policy import draft_features

        K = min(self.k, self.depth.max_depth)
        st = torch.stack(stats, 1)[:, :K] if stats else None
        feats = draft_features(A, K, st, conf[:, :K] if conf is not None else None, self.runner.device)
        p = self.depth.accept_probs(feats)
        live = self.depth.live(p, A)
        if self.depth.host_width is not None:
            self._last_p = p.double().cpu().tolist()  # host copy: live() above read p on the host already
        self.stats["depth_cut"] = self.stats.get("depth_cut", 0) + sum(self.k - v for v in live)
        return live

    def _slot(self, req, p: int) -> int:
        b = req.block_ids
        return b[p // 64] * 64 + p % 64 if p // 64 < len(b) else -1

    def _propose_dflash(self, out, accepted: dict[str, list[int]], defer_tail: bool = False):
        """DFlash: store the context rows this step verified, then draft all k tokens of every
        request that keeps decoding with one block forward."""
        r = self.runner
        dev = r.device
        d = self.dflash
        rows, pos, slots = [], [], []
        t = 0
        for s in out.reqs:
            req, base = s.req, t
            t += s.num_new
            # a verify step keeps the last token and the accepted drafts (acc = accepted + 1 token)
            m = min(len(accepted.get(req.request_id, [])), s.num_new) if s.num_draft else s.num_new
            for j in range(m):
                rows.append(base + j)
                pos.append(s.start + j)
                slots.append(self._slot(req, s.start + j))
        aux = r.model.aux_hidden
        if rows:
            ri = torch.tensor(rows, device=dev)
            states = d.context_states([a.index_select(0, ri) for a in aux])
            d.store_context(states, torch.tensor(pos, device=dev), torch.tensor(slots, device=dev), self.dcaches)
        areqs = [s.req for s in out.reqs
                 if not s.req.status.finished and s.req.num_computed_tokens == s.req.num_tokens - 1]
        if not areqs:
            return
        A = len(areqs)
        last = [q.num_computed_tokens - 1 for q in areqs]
        C = max(last) + 1
        # context slots from the block-table rows on the device (no per-position host work)
        bt = r._to_dev(np.stack([r._bt_row(q) for q in areqs])).long()
        p = torch.arange(C, device=dev)
        lt = torch.tensor(last, device=dev)
        cs = bt[:, (p // 64).clamp(max=bt.shape[1] - 1)] * 64 + p % 64
        ctx_slots = torch.where(p[None] <= lt[:, None], cs, -1)
        bonus = torch.tensor([q.token_at(q.num_computed_tokens) for q in areqs], device=dev)
        h = d(bonus, torch.tensor(last, device=dev), ctx_slots, ctx_slots >= 0, self.dcaches, self.k)
        if defer_tail:
            return areqs, h
        temps_l = [q.params.temperature for q in areqs]
        temps = torch.tensor(temps_l, dtype=torch.float32, device=dev) if any(v > 0 for v in temps_l) else None
        samp = [i for i, v in enumerate(temps_l) if v > 0]
        qbuf = torch.empty(self.k, len(samp), r.model.vocab_local, dtype=torch.float32, device=dev) if samp else None
        drafts, stats = [], []
        for j in range(self.k):
            logits = r.model.compute_logits(h[:, j].contiguous())
            drafts.append(_sample(logits, temps, r.cfg.seed ^ (_SEED_DRAFT + j), r.step_counter, r.model.vocab_offset))
            if self.depth is not None and self.depth.uses_stats:
                stats.append(logit_stats(logits, _all_reduce))
            if samp:
                sel = torch.tensor(samp, device=dev)
                e, ssum = tempered_probs(logits.index_select(0, sel), temps.index_select(0, sel))
                qbuf[j] = e / ssum[:, None]
        live = self._live(A, stats, d.confidence(h) if (self.depth is not None and self.depth.uses_conf) else None)
        dh = torch.stack(drafts, dim=1).cpu().tolist()
        self._set_drafts(areqs, dh, live)
        for qi, a in enumerate(samp):
            self.q_store[areqs[a].request_id] = (qbuf, qi)

    def _ctx(self, pos, tseq, reqs) -> StepContext:
        r = self.runner
        p = np.asarray(pos, dtype=np.int64)
        ts = np.asarray(tseq, dtype=np.int64)
        S = len(reqs)
        cap = r.max_blocks_per_seq * 64
        bt = np.zeros((S, r.max_blocks_per_seq), dtype=np.int32)
        slots = np.full(len(pos), -1, dtype=np.int64)
        for i, req in enumerate(reqs):
            bt[i, : len(req.block_ids)] = req.block_ids
        for i in range(len(pos)):
            b = reqs[ts[i]].block_ids
            if p[i] // 64 < len(b):  # draft positions past the allocated blocks write nothing
                slots[i] = b[p[i] // 64] * 64 + p[i] % 64
        cu = np.zeros(S + 1, dtype=np.int32)
        np.add.at(cu, ts + 1, 1)
        cu = np.cumsum(cu).astype(np.int32)

        def t(a, dt):
            return r._to_dev(np.ascontiguousarray(a, dtype=dt))

        return StepContext(positions=t(p, np.int32), num_tokens=len(pos), slot_mapping=t(slots, np.int64),
                           token_seq=t(ts, np.int32), ctx_lens=t(np.minimum(p + 1, cap), np.int32),
                           block_table=t(bt, np.int32), max_ctx=int(min(p.max() + 1, cap)),
                           cu_seqlens=t(cu, np.int32), kda_slots=t(np.zeros(S), np.int32),
                           has_init=t(np.ones(S), np.int32), mla_caches=r.mla_caches, kda_states=r.kda_states,
                           gqa_caches=r.gqa_caches)

    def acceptance_rate(self) -> float:
        return self.stats["accepted"] / max(1, self.stats["proposed"])
