"""Step runners driven by the worker loop.

A runner turns one decoded step plan (numpy arrays, see runtime/wire.py) into one
SeqStepOutput record per planned sequence.  Two implementations:

* ``CpuReferenceRunner`` -- the fp32 PyTorch reference model, tensor-parallel over
  gloo.  It is the CPU plumbing model: the whole control plane (C++ master, shared
  memory, eventfds, scheduling, prefix caching with recurrent checkpoints, speculative
  verify) runs end to end without a GPU.
* ``GpuRunner`` -- the B200 runner (models/qwen35.py): decode-only plans replay the
  bucket's CUDA graph, other plans run the varlen prefill path; recurrent-state
  checkpoints are snapshotted by the GDN prefill kernel and restored with device copies.

Both implement greedy sampling (global argmax, smallest id on ties) and temperature /
top-k / top-p sampling with a per-sequence seed, identical on every rank.

Reference parity: worker/zstep_worker/models/qwen35_moe.py (launch :1622, finish
:1908, rollback :1861), sampler.py (sample_tp8_logits :127), spec_decode.py
(verify_greedy :41, verify_batch :55).
"""

from __future__ import annotations

import os

import numpy as np
import torch
import torch.distributed as dist

from . import wire
from .runahead import RunAheadGuard, TorchEventBackend
from ..models import sampling_head
from ..sampling import sample_logits, verify_greedy
from ..utils.env import own_process_group_store, runtime_config


def _resolve_config(name: str):
    from ..config import PRESETS, DeepSeekConfig, Qwen35Config

    if name in PRESETS:
        return PRESETS[name]()
    if DeepSeekConfig.is_hf_config(name):
        return DeepSeekConfig.from_hf(name)
    return Qwen35Config.from_hf(name)


def _is_deepseek(cfg) -> bool:
    from ..config import DeepSeekConfig

    return isinstance(cfg, DeepSeekConfig)


def _weights(cfg, name: str, seed: int):
    from ..models.deepseek_weights import DeepSeekRandomWeights
    from ..models.weights import RandomWeights, SafetensorsWeights

    if _is_deepseek(cfg):
        if os.path.isdir(name):
            from ..models.hf_checkpoint import DeepSeekSafetensorsWeights

            return DeepSeekSafetensorsWeights(cfg, name)
        return DeepSeekRandomWeights(cfg, seed=seed)
    if os.path.isdir(name):
        return SafetensorsWeights(cfg, name)
    return RandomWeights(cfg, seed=seed)


def make_runner(args, rank: int, world: int, geo):
    if world > 1 and not dist.is_initialized():
        # This group is hosted by worker rank 0 at MASTER_ADDR/MASTER_PORT, also when the
        # master itself was started under torchrun.
        own_process_group_store()
        backend = "nccl" if args.device == "cuda" else "gloo"
        if args.device == "cuda":
            torch.cuda.set_device(rank % max(1, torch.cuda.device_count()))
        dist.init_process_group(backend, rank=rank, world_size=world)
    if args.model == "micro":
        from ..models.micro import MicroStepRunner

        coll = None
        if args.device == "cuda" and world > 1:
            from ..parallel import make_collectives

            coll = make_collectives(torch.device("cuda", torch.cuda.current_device()))
        return MicroStepRunner(args, rank, world, geo, device=args.device, collectives=coll)
    if args.device == "cpu":
        return CpuReferenceRunner(args, rank, world, geo)
    return GpuRunner(args, rank, world, geo)


def _outputs(n: int) -> np.ndarray:
    out = np.zeros(n, dtype=wire.SEQ_OUTPUT_DTYPE)
    return out


class CpuReferenceRunner:
    """fp32 reference model driven by step plans: one state per request slot, plus
    checkpoint slots (recurrent models) or paged caches rebuilt through the plans' page
    tables (attention-only models, which also serve the host DRAM tier's transfers)."""

    def __init__(self, args, rank: int, world: int, geo):
        from ..models.deepseek_ref import DeepSeekReference
        from ..models.qwen35_ref import Qwen35Reference

        torch.set_num_threads(max(1, (os.cpu_count() or 2) // max(1, world)))
        self.cfg = _resolve_config(args.model)
        self.rank, self.world = rank, world
        ar = (lambda x: self._allreduce(x)) if world > 1 else None
        model_cls = DeepSeekReference if _is_deepseek(self.cfg) else Qwen35Reference
        src = _weights(self.cfg, args.model, args.seed)
        self.model = model_cls(self.cfg, src, device="cpu", quant=False, tp_rank=rank, tp_size=world, allreduce=ar)
        # Model-drafted speculation: K greedy drafts per sampled sequence after each step,
        # from the MTP layer (Qwen3.5) or the DSpark head (DeepSeek).
        self.spec = getattr(args, "spec_method", "none")
        self.num_spec = 0
        if self.spec in ("mtp", "dspark"):
            want = "dspark" if _is_deepseek(self.cfg) else "mtp"
            if self.spec != want or (want == "mtp" and not self.cfg.mtp_num_hidden_layers):
                raise ValueError(f"--spec-method {self.spec} does not fit this model")
            if want == "dspark":
                self.model.load_dspark(src)
            self.num_spec = args.num_spec_tokens
        self.states: dict[int, object] = {}
        self.ckpt: dict[int, object] = {}
        self.generated: dict[int, list[int]] = {}  # per slot: generated tokens (penalties)
        # Attention-only models (DeepSeek-style) also keep their caches paged, like the GPU
        # runner: [layers, pages, page_size, dim] per cache, addressed through the page
        # tables the plans carry.  A sequence's state is rebuilt from its pages at every
        # step, so a prefix shared through the page table, a page reloaded from the host
        # DRAM tier, or a rejected speculative row all behave as on the GPU.
        self.paged = None
        self.dram = None
        if _is_deepseek(self.cfg):
            c = self.cfg
            npg, ps = getattr(args, "num_pages", 256), geo.page_size
            L = c.num_hidden_layers
            self.paged = [torch.zeros(L, npg, ps, c.kv_cache_dim), torch.zeros(L, npg, ps, c.index_head_dim)]
            if self.spec == "dspark":  # the draft layer's own caches, same page table
                self.paged += [torch.zeros(1, npg, ps, c.kv_cache_dim), torch.zeros(1, npg, ps, c.index_head_dim)]
            self.page_size = ps
            self.ptab: dict[int, np.ndarray] = {}
            if getattr(args, "dram_kv_blocks", 0):
                from .kv_dram import DramKvArena

                self.dram = DramKvArena(self.paged, args.dram_kv_blocks)

    def _allreduce(self, x: torch.Tensor) -> torch.Tensor:
        x = x.contiguous()
        dist.all_reduce(x)
        return x

    def _full_logits(self, shard: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return shard
        parts = [torch.empty_like(shard) for _ in range(self.world)]
        dist.all_gather(parts, shard.contiguous())
        return torch.cat(parts)

    # ------------------------------------------------------------------ paged caches
    def _page_of(self, slot: int, p: int) -> int:
        t = self.ptab.get(slot)
        j = p // self.page_size
        return int(t[j]) if t is not None and j < len(t) else 0

    def _state_from_pages(self, slot: int, pos0: int):
        """A fresh state holding rows 0..pos0-1 of the slot's paged caches."""
        st = self.model.new_state()
        if pos0 > 0:
            q = np.arange(pos0)
            pg = torch.as_tensor([self._page_of(slot, int(x)) for x in q], dtype=torch.long)
            off = torch.as_tensor(q % self.page_size, dtype=torch.long)
            for li in range(len(st.ckv)):
                st.ckv[li] = self.paged[0][li, pg, off].clone()
                st.ik[li] = self.paged[1][li, pg, off].clone()
            if len(self.paged) > 2:
                st.dckv = self.paged[2][0, pg, off].clone()
                st.dik = self.paged[3][0, pg, off].clone()
            st.pos = pos0
        return st

    def _rows_to_pages(self, slot: int, st, p: int) -> None:
        pg = self._page_of(slot, p)
        if pg == 0:
            return  # past the sequence's pages (never read back)
        for li in range(len(st.ckv)):
            self.paged[0][li, pg, p % self.page_size] = st.ckv[li][p]
            self.paged[1][li, pg, p % self.page_size] = st.ik[li][p]

    def _draft_rows_to_pages(self, slot: int, st, p0: int) -> None:
        """Draft-layer cache rows p0.. (contexts and the scratch block rows)."""
        if len(self.paged) < 3 or st.dckv is None:
            return
        for p in range(p0, st.dckv.shape[0]):
            pg = self._page_of(slot, p)
            if pg:
                self.paged[2][0, pg, p % self.page_size] = st.dckv[p]
                self.paged[3][0, pg, p % self.page_size] = st.dik[p]

    def execute(self, plan: dict) -> np.ndarray:
        if plan["opcode"] == wire.OP_KV_TRANSFER:
            if self.dram is None:
                raise RuntimeError("KvTransfer step without a DRAM arena (--dram-kv-blocks 0, or a recurrent model)")
            self.dram.transfer(plan["token_ids"], plan["positions"], plan["row_slot"])
            # A demoted page is free: on a GPU its next owner overwrites it.  Poison it here,
            # so a prefix that comes back without its reload diverges instead of reading
            # rows that merely happen to survive.
            down = [int(pg) for pg, up in zip(plan["token_ids"], plan["row_slot"]) if not int(up)]
            if down:
                idx = torch.as_tensor(down, dtype=torch.long)
                for c in self.paged:
                    c[:, idx] = float("nan")
            return _outputs(0)
        n = plan["num_seqs"]
        out = _outputs(n)
        qs, toks, pos = plan["query_start"], plan["token_ids"], plan["positions"]
        ckpt_at = {int(r): int(s) for r, s in zip(plan["ckpt_row"], plan["ckpt_slot"])}
        # A slot's page-table row travels once per request, in the request's first plan:
        # those slots start a new request (a prefix hit may start it past position 0).
        fresh = {int(x) for x in plan["dirty_rows"]}
        if self.paged is not None:
            for k, slot in enumerate(plan["dirty_rows"]):
                self.ptab[int(slot)] = np.array(plan["dirty_pages"][k])
        for i in range(n):
            slot = int(plan["seq_slot"][i])
            r0, r1 = int(qs[i]), int(qs[i + 1])
            if self.paged is not None and r1 > r0:
                self.states[slot] = self._state_from_pages(slot, int(pos[r0]))
            elif int(plan["restore_slot"][i]) >= 0:
                self.states[slot] = self.model.clone_state(self.ckpt[int(plan["restore_slot"][i])])
            if r1 > r0 and int(pos[r0]) == 0:
                self.states[slot] = self.model.new_state()
            if slot in fresh or (r1 > r0 and int(pos[r0]) == 0):
                self.generated[slot] = []  # penalty history of the new request
            st = self.states[slot]
            width = int(plan["spec_width"][i])
            row_logits, row_states, row_hidden = [], [], []
            for r in range(r0, r1):
                assert st.pos == int(pos[r]), f"slot {slot}: state at {st.pos}, plan position {int(pos[r])}"
                lg = self.model.step(st, int(toks[r]))
                if self.paged is not None:
                    self._rows_to_pages(slot, st, int(pos[r]))
                if self.num_spec:
                    row_hidden.append(self.model.last_aux if self.spec == "dspark" else st.hidden)
                if r in ckpt_at:
                    self.ckpt[ckpt_at[r]] = self.model.clone_state(st)
                if width > 0:
                    row_logits.append(self._full_logits(lg))
                    row_states.append(self.model.clone_state(st))
                elif r == r1 - 1 and int(plan["sample_row"][i]) >= 0:
                    row_logits.append(self._full_logits(lg))
            out[i]["req_slot"] = slot
            if int(plan["sample_row"][i]) < 0:
                if self.num_spec:  # prefill chunk: draft-model state for its rows, no drafts
                    self._draft(self.states[slot], [int(t) for t in toks[r0 + 1:r1]], row_hidden, int(pos[r0]), 0)
                    if self.paged is not None:
                        self._draft_rows_to_pages(slot, self.states[slot], int(pos[r0]))
                continue
            sp = plan["sampling"][i]
            if width > 0:
                drafts = [int(t) for t in toks[r0 + 1:r1]]
                targets = [sample_logits(l, sp) for l in row_logits]
                acc = verify_greedy(drafts, targets)  # accepted drafts + bonus token
                # Roll the state back to the last accepted row.
                self.states[slot] = row_states[len(acc) - 1]
                tokens = acc
            else:
                hist = self.generated.setdefault(slot, [])[-4096:]
                tokens = [sample_logits(row_logits[-1], sp, hist)]
                if int(sp["logprobs"]) >= 0:
                    lsm = torch.log_softmax(row_logits[-1].double(), dim=0)
                    out[i]["logprobs"][0] = float(lsm[tokens[0]])
                    k = min(int(sp["logprobs"]), len(out[i]["top_ids"]))
                    if k > 0:
                        top = torch.topk(row_logits[-1].float(), k)
                        out[i]["top_ids"][:k] = top.indices.numpy()
                        out[i]["top_logprobs"][:k] = lsm[top.indices].numpy()
            self.generated.setdefault(slot, []).extend(tokens)
            out[i]["num_tokens"] = len(tokens)
            out[i]["tokens"][:len(tokens)] = tokens
            if self.num_spec:
                # Row r0+j is followed by the prompt / draft token r0+j+1 (non-verify rows) or by
                # the target's token acc[j] (verify rows, accepted prefix only).
                if width > 0:
                    nxt, hid = tokens, row_hidden[:len(tokens)]
                else:
                    nxt, hid = [int(t) for t in toks[r0 + 1:r1]] + tokens[:1], row_hidden
                d = self._draft(self.states[slot], nxt, hid, int(pos[r0]), self.num_spec)
                if self.paged is not None:
                    self._draft_rows_to_pages(slot, self.states[slot], int(pos[r0]))
                out[i]["next_drafts"][:len(d)] = d
                out[i]["num_drafts"] = len(d)
        return out

    def _draft(self, st, next_tokens: list[int], hidden: list, pos0: int, num_drafts: int) -> list[int]:
        """Draft-model catch-up for the target rows pos0.. (``next_tokens[j]`` follows row j,
        ``hidden[j]`` is its hidden state, or its auxiliary FFN inputs for DSpark), then
        ``num_drafts`` greedy drafts after the last of ``next_tokens``."""
        if self.spec == "dspark":
            # DSpark contexts need no following token: every row of the chunk gets one.
            for j, aux in enumerate(hidden):
                self.model.dspark_context(st, aux, pos0 + j)
            if not num_drafts or not next_tokens:
                return []
            return self.model.dspark_draft(st, next_tokens[-1], pos0 + len(next_tokens), num_drafts,
                                           self._full_logits)
        lg = h = None
        for j, tok in enumerate(next_tokens):
            lg, h = self.model.mtp_step(st, tok, hidden[j], pos0 + j)
        drafts = []
        p = pos0 + len(next_tokens)
        for _ in range(num_drafts if lg is not None else 0):
            d = int(torch.argmax(self._full_logits(lg)))
            drafts.append(d)
            if len(drafts) == num_drafts:
                break
            lg, h = self.model.mtp_step(st, d, h, p)
            p += 1
        return drafts

    def close(self) -> None:
        if dist.is_initialized():
            dist.destroy_process_group()


class GpuRunner:
    """B200 runner: the kernels of models/qwen35.py driven by step plans."""

    # Defaults for every attribute ``execute`` reads, so a runner built by ``wrap`` (no CLI
    # arguments) behaves like one built by the worker.
    nvtx = False
    head = None
    dram = None
    rank = 0
    guard = RunAheadGuard(0)  # eager-step run-ahead cap (off unless the worker sets one)

    @classmethod
    def wrap(cls, model_runner, rank: int = 0, nvtx: bool = False) -> "GpuRunner":
        """A step-plan runner around an already built model runner (Qwen35Runner or
        DeepSeekRunner): what the worker builds, minus argument parsing, weight loading and
        the DRAM arena.  Tests and embedders drive plans through this."""
        g = cls.__new__(cls)
        g.r, g.rank, g.nvtx = model_runner, rank, nvtx
        g.head = None
        g.dram = None
        g.dev = model_runner.dev
        g.cfg = model_runner.cfg
        return g

    def __init__(self, args, rank: int, world: int, geo):
        from ..models.deepseek import DeepSeekRunner
        from ..models.qwen35 import Qwen35Runner
        from ..parallel import make_collectives

        self.cfg = _resolve_config(args.model)
        self.dev = torch.device("cuda", torch.cuda.current_device())
        self.nvtx = runtime_config().nvtx
        self.guard = RunAheadGuard(runtime_config().runahead_depth, TorchEventBackend(self.dev))
        coll = make_collectives(self.dev) if world > 1 else None
        # Model-drafted speculation: the MTP head for Qwen3.5, the DSpark head for DeepSeek.
        want = "dspark" if _is_deepseek(self.cfg) else "mtp"
        if args.spec_method in ("mtp", "dspark") and args.spec_method != want:
            raise ValueError(f"--speculative-method {args.spec_method} does not fit this model (use {want})")
        num_spec = args.num_spec_tokens if args.spec_method == want else 0
        runner_cls = DeepSeekRunner if _is_deepseek(self.cfg) else Qwen35Runner
        self.r = runner_cls(self.cfg, device=self.dev, weights=_weights(self.cfg, args.model, args.seed),
                              max_seqs=geo.max_seqs, max_prefill_tokens=geo.max_step_tokens,
                              num_pages=args.num_pages, page_size=geo.page_size, max_model_len=args.max_model_len,
                              num_ckpt_slots=args.num_ckpt_slots, tp_rank=rank, tp_size=world, collectives=coll,
                              seed=args.seed, num_spec_tokens=num_spec)
        self.rank = rank
        self.head = None  # full-distribution sampling head, created on first use
        self.dram = None
        if getattr(args, "dram_kv_blocks", 0):
            from .kv_dram import DramKvArena

            self.dram = DramKvArena(self.r.paged_caches(), args.dram_kv_blocks)

    def execute(self, plan: dict) -> np.ndarray:
        """One step plan.  With ZSTEP_NVTX=1 the step is an NVTX range named after its kind
        (decode / prefill / verify / kv-transfer), for Nsight timelines."""
        if not self.nvtx:
            return self._execute(plan)
        kind = ("kv-transfer" if plan["opcode"] == wire.OP_KV_TRANSFER else
                "verify" if plan["flags"] & wire.FLAG_SPEC_VERIFY else
                "decode" if plan["flags"] & wire.FLAG_DECODE_ONLY else "prefill")
        torch.cuda.nvtx.range_push(f"zstep {kind} rows={int(plan['num_rows'])}")
        try:
            return self._execute(plan)
        finally:
            torch.cuda.nvtx.range_pop()

    def _execute(self, plan: dict) -> np.ndarray:
        r = self.r
        n = plan["num_seqs"]
        if plan["opcode"] == wire.OP_KV_TRANSFER:
            if self.dram is None:
                raise RuntimeError("KvTransfer step without a DRAM arena (--dram-kv-blocks 0)")
            self.dram.transfer(plan["token_ids"], plan["positions"], plan["row_slot"])
            return _outputs(0)
        out = _outputs(n)
        for k, slot in enumerate(plan["dirty_rows"]):
            r.page_table[int(slot)].copy_(torch.from_numpy(plan["dirty_pages"][k][: r.max_pages]).to(r.dev))
        for i in range(n):
            src = int(plan["restore_slot"][i])
            if src >= 0:
                r.copy_recurrent_state(src, int(plan["seq_slot"][i]))
        rows = plan["num_rows"]
        if r.spec is not None:
            return self._execute_spec(plan, n, out)
        sampling = bool(plan["flags"] & wire.FLAG_SAMPLING)
        decode_only = bool(plan["flags"] & wire.FLAG_DECODE_ONLY)
        if sampling:
            # Temperature sampling runs inside the lm_head GEMM (Gumbel-perturbed argmax);
            # the per-sequence seed plus the row position make it reproducible.
            sp = plan["sampling"]
            r.set_sampling([float(sp[i]["temperature"]) for i in range(n)], [int(sp[i]["seed"]) for i in range(n)])
            self._sampling_set = True
        elif getattr(self, "_sampling_set", False):
            r.clear_sampling()
            self._sampling_set = False
        qs, pos = plan["query_start"], plan["positions"]
        # New requests: a slot whose page-table row this plan carries (sent once, with the
        # request's first chunk, also when a prefix hit starts it past position 0) or a
        # chunk starting at position 0.  Their penalty rings restart.
        fresh = {int(x) for x in plan["dirty_rows"]}
        starting = [int(plan["seq_slot"][i]) for i in range(n)
                    if int(plan["seq_slot"][i]) in fresh or (qs[i + 1] > qs[i] and int(pos[qs[i]]) == 0)]
        full = sampling_head.needs_full(plan["sampling"], n)
        if full and self.head is None:
            self.head = sampling_head.SamplingHead(r)
        if self.head is not None:
            self.head.reset(starting)
        if decode_only:
            r.stage(plan["token_ids"], plan["positions"], plan["row_slot"])
            ids = r.decode_step(rows).cpu().numpy()
            lm_in = (r.buf["xq"], r.buf["xsf"])
        else:
            seq_start = plan["query_start"].tolist()
            r.stage(plan["token_ids"], plan["positions"], plan["row_slot"], seq_start=seq_start)
            ck = None
            if len(plan["ckpt_row"]):
                ck = r.checkpoint_args(plan["ckpt_row"], plan["ckpt_slot"], plan["query_start"])
            self.guard.before_launch()
            dev_ids = r.prefill_forward(rows, n, ckpt=ck)
            self.guard.after_launch()
            ids = dev_ids.cpu().numpy()
            lm_in = (r.buf["xq_last"], r.last_lm_sf)
        lp = tids = tlps = None
        if full:
            # Top-k / top-p / penalties / logprobs: f32 lm_head over the same normed rows and
            # the full-distribution sampling kernel.
            record = [int(plan["sample_row"][i]) >= 0 for i in range(n)]
            top_n = int(max(0, plan["sampling"]["logprobs"][:n].max()))
            ids, lp, tids, tlps = self.head.sample(n, lm_in[0], lm_in[1], plan["seq_slot"], plan["sampling"],
                                                   top_n=top_n, record=record)
        for i in range(n):
            out[i]["req_slot"] = int(plan["seq_slot"][i])
            if int(plan["sample_row"][i]) >= 0:
                out[i]["num_tokens"] = 1
                out[i]["tokens"][0] = int(ids[i])
                if lp is not None:
                    out[i]["logprobs"][0] = float(lp[i])
                    k = max(0, int(plan["sampling"]["logprobs"][i]))
                    out[i]["top_ids"][:k] = tids[i, :k]
                    out[i]["top_logprobs"][:k] = tlps[i, :k]
        return out

    def _execute_spec(self, plan: dict, n: int, out):
        """Steps of an engine with MTP speculative decoding (eager): one varlen target forward
        over all rows (verify rows of drafting sequences included), greedy acceptance,
        recurrent-state replay of the accepted rows, then MTP drafts for the next step."""
        r = self.r
        rows = plan["num_rows"]
        K = r.num_spec
        if (runtime_config().decode_graphs and n > 0 and rows == n * (K + 1) and not len(plan["ckpt_row"])
                and not plan["flags"] & wire.FLAG_SAMPLING
                and all(int(w) == K + 1 for w in plan["spec_width"][:n])
                and all(int(q) == i * (K + 1) for i, q in enumerate(plan["query_start"][:n + 1]))
                and all(int(sr) == (i + 1) * (K + 1) - 1 for i, sr in enumerate(plan["sample_row"][:n]))):
            nb = r.spec.graph_bucket(n) if hasattr(r.spec, "graph_bucket") else None
            if nb is not None:
                return self._execute_spec_graph(plan, n, nb, out)
        qs = plan["query_start"].tolist()
        ids = plan["token_ids"][:rows].tolist()
        pos = plan["positions"][:rows].tolist()
        rslot = plan["row_slot"][:rows].tolist()
        sw = plan["spec_width"][:n].tolist()
        srow = plan["sample_row"][:n].tolist()
        r.stage(ids, pos, rslot, seq_start=qs[:n + 1])
        lm_rows, seq_lm, verify_slots = [], [], []
        for i in range(n):
            r0, r1 = qs[i], qs[i + 1]
            if sw[i] > 0:
                seq_lm.append((len(lm_rows), r1 - r0))
                lm_rows.extend(range(r0, r1))
                verify_slots.append(r.spec_slot_base + int(plan["seq_slot"][i]))
            elif srow[i] >= 0:
                seq_lm.append((len(lm_rows), 1))
                lm_rows.append(r1 - 1)
                verify_slots.append(None)
            else:
                seq_lm.append(None)
                verify_slots.append(None)
        ck = None
        if len(plan["ckpt_row"]):
            ck = r.checkpoint_args(plan["ckpt_row"], plan["ckpt_slot"], plan["query_start"])
        lm_t = torch.tensor(lm_rows, dtype=torch.long, device=r.dev)
        targets = r.spec.forward(rows, n, lm_t, verify_slots, ckpt=ck).cpu().tolist() if lm_rows else []
        replay, replay_slots, replay_pos = [], [], []
        m_ids, m_pos, m_slot, m_rows, last_of_seq, drafting = [], [], [], [], [], []
        for i in range(n):
            r0, r1 = qs[i], qs[i + 1]
            out[i]["req_slot"] = int(plan["seq_slot"][i])
            if seq_lm[i] is None:  # prefill chunk that does not sample: draft-model catch-up only
                # An MTP entry needs the token after its row (unknown for the chunk's last
                # row); a DSpark context needs only the row itself.
                end = r1 if r.spec.context_only else r1 - 1
                for rr in range(r0, end):
                    nxt = ids[rr + 1] if rr + 1 < r1 else 0
                    m_ids.append(nxt), m_pos.append(pos[rr]), m_slot.append(rslot[rr]), m_rows.append(rr)
                continue
            st, cnt = seq_lm[i]
            t = targets[st:st + cnt]
            if sw[i] > 0:
                drafts = ids[r0 + 1:r1]
                acc = []
                for j, d in enumerate(drafts):
                    if t[j] != d:
                        acc.append(t[j])
                        break
                    acc.append(d)
                else:
                    acc.append(t[len(drafts)])
                replay.append((r0, len(acc)))
                replay_slots.append(rslot[r0])
                replay_pos.append(pos[r0])
                for j, tok in enumerate(acc):  # the target token after row r0+j is acc[j]
                    m_ids.append(tok), m_pos.append(pos[r0 + j]), m_slot.append(rslot[r0]), m_rows.append(r0 + j)
            else:
                acc = [t[0]]
                for rr in range(r0, r1):
                    nxt = ids[rr + 1] if rr + 1 < r1 else acc[0]
                    m_ids.append(nxt), m_pos.append(pos[rr]), m_slot.append(rslot[rr]), m_rows.append(rr)
            out[i]["num_tokens"] = len(acc)
            out[i]["tokens"][:len(acc)] = acc
            last_of_seq.append(len(m_ids) - 1)
            drafting.append(i)
        r.spec.replay(replay, replay_slots, replay_pos)
        if m_ids:
            rows_t = torch.tensor(m_rows, dtype=torch.long, device=r.dev)
            if drafting:
                drafts = r.spec.draft(m_ids, m_pos, m_slot, rows_t, last_of_seq)
                for k, i in enumerate(drafting):
                    out[i]["next_drafts"][:len(drafts[k])] = drafts[k]
                    out[i]["num_drafts"] = len(drafts[k])
            else:
                r.spec.catch_up(m_ids, m_pos, m_slot, rows_t)
        return out

    def _execute_spec_graph(self, plan: dict, n: int, nb: int, out):
        """A steady-state verify step (every sequence: last token + K drafts, greedy) as one
        CUDA-graph replay: verify, acceptance, state roll-back and the next drafts all run on
        the device; the host reads one [n, 2K+2] record per step."""
        r = self.r
        K = r.num_spec
        K1 = K + 1
        R, rows = nb * K1, plan["num_rows"]
        ids = np.zeros(R, np.int32)
        pos = np.ones(R, np.int32)
        slot = np.full(R, r.dummy_slot, np.int32)
        ids[:rows] = plan["token_ids"][:rows]
        pos[:rows] = plan["positions"][:rows]
        slot[:rows] = plan["row_slot"][:rows]
        r.stage(ids, pos, slot, seq_start=[i * K1 for i in range(nb + 1)])
        spare = [r.spec_slot_base + int(plan["seq_slot"][i]) for i in range(n)] + [r.dummy_slot] * (nb - n)
        r.spec.out_slots[:nb].copy_(torch.tensor(spare, dtype=torch.int32))
        r.spec.run_verify_graph(nb)
        rec = r.spec.g_record[:n].cpu().numpy()
        for i in range(n):
            acc = int(rec[i, 0])
            out[i]["req_slot"] = int(plan["seq_slot"][i])
            out[i]["num_tokens"] = acc
            out[i]["tokens"][:acc] = rec[i, 1:1 + acc]
            out[i]["next_drafts"][:K] = rec[i, K + 2:2 * K + 2]
            out[i]["num_drafts"] = K
        return out

    def close(self) -> None:
        torch.cuda.synchronize()
        if dist.is_initialized():
            dist.destroy_process_group()
