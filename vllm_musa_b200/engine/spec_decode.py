"""Model-based speculative proposers.

The layer drafters are one extra decoder layer fed by the target's own features:
``MTPDrafter`` drives DeepSeek's multi-token-prediction layer (the checkpoint's layer
``num_layers``), ``EagleDrafter`` an EAGLE head over a dense decoder (``models/eagle.py``),
``Eagle3Drafter`` an EAGLE-3 head reading three of the target's residual streams.
``MedusaDrafter`` needs no layer: its heads read the final hidden state only.
After every engine step the drafter runs its layer over each request's positions whose next
token is now known: position p combines the embedding of token p+1 with the main model's final
hidden state at p, writes the draft layer's KV for p (extra cache layer ``num_layers``, same
block table and slots as the main model), and its logits predict token p+2.  The prediction
made at the position just before the request's pending token becomes the draft the scheduler
verifies in the next step (exact acceptance, see csrc/runtime/scheduler.cpp); with a tree
width w > 1 the top w predictions are verified together as sibling nodes of a token tree, and
the hidden state of the accepted node feeds the next draft.  With ``num_speculative_tokens``
k > 1 the layer then runs k - 1 more single-token steps on its own output (chained drafts,
KV slots reserved ahead of verification).  Positions of rejected drafts are skipped: their
main-model KV and hidden states are stale and get overwritten.

Reference counterparts: vllm_musa/v1/spec_decode/utils.py:4-124 (eagle / MTP input
preparation kernels) and patches/vllm__v1__spec_decode__eagle.patch.py (drafter wiring).
"""
from __future__ import annotations

import torch

from ..attention.metadata import AttnMetadata


class ModelDrafter:
    """Drafts from a draft layer (one, or a chain of ``num_tokens`` fed back through the layer):
    ``forward(ids, prev_hidden, meta, kv_caches)`` ->
    hidden rows, ``logits(hidden)`` -> this rank's vocab shard of the draft logits."""

    def __init__(self, engine, forward, logits, num_tokens: int = 1, tree_width: int = 1,
                 features=None, pick=None):
        if num_tokens < 1:
            raise ValueError("num_speculative_tokens must be >= 1")
        if num_tokens > 1 and tree_width > 1:
            raise ValueError("chained drafts (num_speculative_tokens > 1) are verified as a "
                             "chain: token trees take one draft level")
        self.k = num_tokens
        self.engine = engine
        self.model = engine.model
        self.runner = engine.runner
        self.forward = forward
        self.logits = logits
        self.tree_width = tree_width  # > 1: the top tree_width tokens, verified as siblings
        self.proposed = 0
        # per-step-row features the head reads (default: the target's final hidden states)
        self.features = features or (lambda: self.runner.last_hidden)
        # logits -> [S, k] target token ids (default: the target's vocab-parallel sampler)
        self.pick = pick

    def propose(self, scheduler) -> None:
        """Drafts were set right after the previous step; nothing to do before scheduling."""

    @torch.no_grad()
    def after_step(self, plan, sampled) -> None:
        sch = self.engine.scheduler
        b = self.runner.buf
        h = b.h
        hidden = self.features()
        if hidden is None or plan.num_reqs == 0:
            return
        cu = h["cu_q"][:plan.num_reqs + 1].tolist()
        pos_all = h["positions"][:plan.num_tokens]
        # rows: step rows whose KV slot now holds positions start.. (consecutive after the
        # accepted path of a draft tree was compacted); hid_rows: the rows that computed them
        rows, hid_rows, pos, next_ids, cus, lens, req_rows, who = [], [], [], [], [0], [], [], []
        for i, rid in enumerate(plan.req_ids):
            n_tok = sch.num_tokens(rid)
            if n_tok == 0:
                continue  # finished and forgotten
            start = int(pos_all[cu[i]])
            q = cu[i + 1] - cu[i]
            last = min(start + q - 1, n_tok - 2)  # positions whose next token is known
            if last < start:
                continue
            n = last - start + 1
            nxt = sch.tokens_range(rid, start + 1, n)
            rows.extend(range(cu[i], cu[i] + n))
            path = sch.last_path(rid) if plan.tree else []
            if path:
                hid_rows.extend([cu[i]] + [cu[i] + 1 + j for j in path[:n - 1]])
            else:
                hid_rows.extend(range(cu[i], cu[i] + n))
            pos.extend(range(start, start + n))
            next_ids.extend(nxt)
            cus.append(cus[-1] + len(nxt))
            lens.append(last + 1)
            req_rows.append(i)
            who.append((rid, last == n_tok - 2))
        if not rows:
            return
        dev = hidden.device
        rows_t = torch.tensor(rows, dtype=torch.long, device=dev)
        T = len(rows)
        ids = torch.tensor(next_ids, dtype=torch.int32, device=dev)
        positions = torch.tensor(pos, dtype=torch.int32, device=dev)
        slots = b.d["slot_mapping"][:plan.num_tokens][rows_t].contiguous()
        rr = torch.tensor(req_rows, dtype=torch.long, device=dev)
        bt = b.bt2d()[:plan.num_reqs][rr].contiguous()
        cu_t = torch.tensor(cus, dtype=torch.int32, device=dev)
        sl = torch.tensor(lens, dtype=torch.int32, device=dev)
        R = len(req_rows)
        meta = AttnMetadata(T, 0, R, positions, slots, sl, bt, cu_t, max_seq_len=max(lens),
                            tile_scratch=self.runner.tile_scratch,
                            state_slots=b.d["state_slots"][:R])
        prev = hidden[torch.tensor(hid_rows, dtype=torch.long, device=dev)]
        x, xc = self._run(ids, prev, meta)
        last_rows = torch.tensor([c - 1 for c in cus[1:]], dtype=torch.long, device=dev)
        logits = self.logits(x[last_rows])
        if self.k > 1:
            ready = [j for j, (_, r) in enumerate(who) if r]
            if ready:
                sel = torch.tensor(ready, dtype=torch.long, device=dev)
                first = self._greedy(logits.index_select(0, sel))
                self._chain([who[j][0] for j in ready], [lens[j] + 1 for j in ready], first,
                            xc[last_rows].index_select(0, sel))
            return
        if self.pick is not None:  # the head's own vocabulary, whole on this rank
            top = self.pick(logits, self.tree_width).cpu().tolist()
            for k, (rid, ready) in enumerate(who):
                if not ready:
                    continue
                if self.tree_width > 1:
                    sch.set_draft_tree(rid, [int(t) for t in top[k]], [-1] * self.tree_width)
                else:
                    sch.set_draft(rid, [int(top[k][0])])
                self.proposed += self.tree_width
            return
        if self.tree_width > 1:
            smp = self.runner.sampler
            if smp.tp > 1:  # vocab-sharded rows: the full distribution
                logits = smp.comm.all_gather(logits, dim=1)
            logits = logits[:, :self.model.cfg.vocab_size]
            top = torch.topk(logits.float(), self.tree_width, dim=-1).indices.cpu().tolist()
            for k, (rid, ready) in enumerate(who):
                if ready:
                    sch.set_draft_tree(rid, [int(t) for t in top[k]], [-1] * self.tree_width)
                    self.proposed += self.tree_width
            return
        draft = self.runner.sampler(logits, None, None, None, None, None, None).cpu().tolist()
        for k, (rid, ready) in enumerate(who):
            if ready:
                sch.set_draft(rid, [int(draft[k])])
                self.proposed += 1


    def _run(self, ids, prev, meta):
        """The head's forward -> (hidden for its logits, hidden that feeds a chained step)."""
        out = self.forward(ids, prev, meta, self.runner.kv_caches)
        return out if isinstance(out, tuple) else (out, out)

    def _greedy(self, logits) -> list:
        """Most likely target token id of each row."""
        if self.pick is not None:
            return [int(t) for t in self.pick(logits, 1)[:, 0].cpu().tolist()]
        return [int(t) for t in
                self.runner.sampler(logits, None, None, None, None, None, None).cpu().tolist()]

    def _chain(self, rids, n_toks, first, h) -> None:
        """Drafts 2..k: step j runs the head once per request at position n_tok - 2 + j on the
        previous draft token, fed with its own previous output instead of the target's (not yet
        computed) hidden state, writing its layer's K/V at that position's slot (reserved here);
        a request whose slot cannot be reserved keeps the drafts it has."""
        sch = self.engine.scheduler
        dev = h.device
        drafts = {rid: [t] for rid, t in zip(rids, first)}
        live = list(range(len(rids)))
        width = self.runner.max_blocks
        for j in range(1, self.k):
            keep, pos, slots, tables = [], [], [], []
            for i in live:
                p = n_toks[i] - 2 + j
                slot = sch.reserve_slots(rids[i], p, 1)[0]
                if slot < 0:
                    continue
                blocks = list(sch.block_ids(rids[i]))[:width]
                keep.append(i)
                pos.append(p)
                slots.append(slot)
                tables.append(blocks + [0] * (width - len(blocks)))
            if not keep:
                break
            R = len(keep)
            idx = torch.tensor([live.index(i) for i in keep], dtype=torch.long, device=dev)
            h = h.index_select(0, idx)
            ids = torch.tensor([drafts[rids[i]][-1] for i in keep], dtype=torch.int32, device=dev)
            meta = AttnMetadata(R, 0, R, torch.tensor(pos, dtype=torch.int32, device=dev),
                                torch.tensor(slots, dtype=torch.int32, device=dev),
                                torch.tensor([p + 1 for p in pos], dtype=torch.int32, device=dev),
                                torch.tensor(tables, dtype=torch.int32, device=dev),
                                torch.arange(R + 1, dtype=torch.int32, device=dev),
                                max_seq_len=max(pos) + 1, tile_scratch=self.runner.tile_scratch,
                                state_slots=self.runner.buf.d["state_slots"][:R])
            x, h = self._run(ids, h, meta)
            for i, t in zip(keep, self._greedy(self.logits(x))):
                drafts[rids[i]].append(t)
            live = keep
        for rid in rids:
            sch.set_draft(rid, drafts[rid])
            self.proposed += len(drafts[rid])


class MTPDrafter(ModelDrafter):
    def __init__(self, engine, num_tokens: int = 1, tree_width: int = 1):
        model = engine.model
        if getattr(model, "mtp", None) is None:
            raise ValueError("speculative method 'mtp' needs a checkpoint with an MTP layer "
                             "(num_nextn_predict_layers > 0)")
        n = model.cfg.num_layers
        super().__init__(engine, lambda ids, prev, meta, kv: model.forward_mtp(ids, prev, meta,
                                                                              kv[n]),
                         model.compute_logits_mtp, num_tokens, tree_width)


class EagleDrafter(ModelDrafter):
    def __init__(self, engine, num_tokens: int = 1, tree_width: int = 1):
        head = getattr(engine.model, "draft_head", None)
        if head is None:
            raise ValueError("speculative method 'eagle' needs an EAGLE head on the model")
        super().__init__(engine, head.forward_draft, head.compute_logits, num_tokens,
                         tree_width)


class Eagle3Drafter(ModelDrafter):
    """EAGLE-3: the head reads three of the target's residual streams per position (recorded
    by the model into ``aux_buf`` during its forward, graph replays included) and drafts from
    its own vocabulary, mapped to target ids."""

    def __init__(self, engine, num_tokens: int = 1, tree_width: int = 1):
        head = getattr(engine.model, "draft_head", None)
        if head is None or getattr(engine.model, "aux_buf", None) is None:
            raise ValueError("speculative method 'eagle3' needs an EAGLE-3 head on the model")
        super().__init__(engine, head.forward_draft, head.compute_logits, num_tokens,
                         tree_width, features=lambda: engine.model.aux_buf, pick=head.pick)


class MedusaDrafter:
    """Medusa drafts right after every step, from the target's final hidden state at the
    position whose next token is the pending one (``models/medusa.py``): a chain of each head's
    argmax, or with ``tree_width`` w > 1 a token tree filled level by level."""

    def __init__(self, engine, num_tokens: int, tree_width: int = 1):
        self.engine = engine
        self.runner = engine.runner
        self.heads = engine.model.medusa
        self.budget = min(num_tokens, 63)
        self.w = tree_width
        self.proposed = 0

    def propose(self, scheduler) -> None:
        """Drafts were set right after the previous step."""

    @torch.no_grad()
    def after_step(self, plan, sampled) -> None:
        sch = self.engine.scheduler
        hidden = self.runner.last_hidden
        if hidden is None or plan.num_reqs == 0:
            return
        h = self.runner.buf.h
        cu = h["cu_q"][:plan.num_reqs + 1].tolist()
        pos_all = h["positions"][:plan.num_tokens]
        rows, rids = [], []
        for i, rid in enumerate(plan.req_ids):
            n_tok = sch.num_tokens(rid)
            if n_tok == 0:
                continue
            start, q = int(pos_all[cu[i]]), cu[i + 1] - cu[i]
            p = n_tok - 2  # its next token is the pending one
            if not start <= p < start + q:
                continue  # a prompt chunk that does not reach the end of the prompt
            m = p - start
            path = sch.last_path(rid) if plan.tree else []
            rows.append(cu[i] if m == 0 else (cu[i] + 1 + path[m - 1] if path else cu[i] + m))
            rids.append(rid)
        if not rows:
            return
        r = torch.tensor(rows, dtype=torch.long, device=hidden.device)
        logits = self.heads.logits(hidden.index_select(0, r))
        if self.w == 1:
            d = torch.stack([lg.argmax(-1) for lg in logits], 1)[:, :self.budget].cpu().tolist()
            for rid, toks in zip(rids, d):
                sch.set_draft(rid, [int(t) for t in toks])
                self.proposed += len(toks)
            return
        tops = [torch.topk(lg, self.w, dim=-1).indices.cpu().tolist() for lg in logits]
        for n, rid in enumerate(rids):
            toks, par, level = [], [], [-1]
            for depth, top in enumerate(tops):
                nxt = []
                for parent in level:
                    for t in top[n]:
                        if len(toks) == self.budget:
                            break
                        toks.append(int(t))
                        par.append(parent)
                        nxt.append(len(toks) - 1)
                level = nxt
                if len(toks) == self.budget or not level:
                    break
            sch.set_draft_tree(rid, toks, par)
            self.proposed += len(toks)
