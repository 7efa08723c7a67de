"""B200 training update for the reversible models (the benchmark's "step").

One update = `accumulation` microsteps of the reference trainer loop
(scripts/train_baseline.py:247-285): forward, sum cross-entropy / update
targets, reconstruction backward, gradient accumulation; then the global-norm
clip, the warm-up/cosine learning rate and AdamW(0.9, 0.95, wd 0.1).

Layout in HBM (all fixed at construction, so an update can be captured once in
a CUDA graph and replayed):
  - `flat`   fp32 [P]   every parameter (named_parameters order; the tied
                         head/embedding once); module parameters are views
  - `flat_c` bf16 [P]   compute copy, refreshed after each optimizer step;
                         the GEMM weights and the head are views into it
  - `gflat`  fp32 [P]   gradients; layer i's six gradients are contiguous, so
                         each layer is one data-parallel all-reduce bucket
  - logits   bf16 [B*T, Vpad]  the microstep's vocabulary logits (bf16 runs:
                         exp(logit - max of its 128-column block)); Vpad = V
                         rounded up to 64 so every row starts 16-byte aligned
                         for TMA
  - head_stats fp32 [B*T, 2*ceil(V/256), 2]  per-row partial (max, sum exp)
                         pairs written by the head GEMM's epilogue
Per microstep: embedding gather, the fused stack forward, final norm, head GEMM
with the log-sum-exp partials in its epilogue, per-row loss, head dgrad/wgrad
that form dlogits = (softmax - onehot) / targets from the logits inside the
GEMM (fp32 runs: head GEMM, cross-entropy forward+backward in place, plain
dgrad/wgrad), final-norm backward, fused reconstruction backward (engine.py),
deterministic embedding scatter. Every gradient is bitwise reproducible.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import _lib, engine, functional as fn
from .dist import GradBuckets
from .reversible import ReversibleLM

F32 = torch.float32


@dataclass
class TrainSettings:
    """Optimisation fields of configs/midpoint.json (plus the cfg2 batch shape)."""
    batch_size: int = 29
    sequence_length: int = 512
    accumulation: int = 2
    learning_rate: float = 6e-4
    min_learning_rate: float = 6e-5
    warmup_targets: int = 1_000_000
    max_train_targets: int = 50_000_000
    weight_decay: float = 0.1
    beta1: float = 0.9
    beta2: float = 0.95
    grad_clip: float = 1.0
    precision: str = "bf16"
    norm_eps: float | None = 1e-6
    mlp_tokens: int = 0
    fused_head: bool = True  # bf16/f16: cross-entropy inside the head GEMMs (rk_head_*)
    overlap_wgrad: bool = True  # layer weight gradients on a side stream during the reverse sweep
    overlap_forward: bool = True  # microstep m+1's forward sweep beside microstep m's backward
    tied_split: bool = True  # data parallel: the head's share of the tied gradient reduced beside the sweep
    # where microstep m+1's forward sweep starts: at the start of the update,
    # beside microstep 0's forward sweep ("start"; measured fastest), beside
    # microstep m's head GEMM ("head"), or once that GEMM is issued, beside the
    # rest of the head and the reverse sweep ("after_head")
    forward_overlap: str = "start"


def learning_rate(s: TrainSettings, committed: int, update_targets: int) -> float:
    """train_baseline.py:273-277."""
    progress = (committed + update_targets) / s.max_train_targets
    warmup = min(1.0, (committed + update_targets) / s.warmup_targets)
    cosine = s.min_learning_rate + 0.5 * (s.learning_rate - s.min_learning_rate) * (1 + math.cos(math.pi * progress))
    return min(s.learning_rate * warmup, cosine)


class ReversibleTrainer:
    def __init__(self, model: ReversibleLM, settings: TrainSettings, process_group=None):
        if not isinstance(model, ReversibleLM):
            raise ValueError("ReversibleTrainer trains ReversibleLM models")
        dev = next(model.parameters()).device
        fn.require_cuda(next(model.parameters()))
        self.model, self.s, self.dev = model, settings, dev
        self.cfg = model.config
        self.pg = process_group
        self.world = dist.get_world_size(process_group) if process_group is not None else 1
        self.cd = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[settings.precision]
        if settings.norm_eps is not None:
            for m in model.modules():
                if isinstance(m, torch.nn.RMSNorm):
                    m.eps = settings.norm_eps
        # ---- flat parameter / gradient layout
        named = list(model.named_parameters())
        total = sum(p.numel() for _, p in named)
        self.flat = torch.empty(total, device=dev, dtype=F32)
        self.gflat = torch.zeros(total, device=dev, dtype=F32)
        self.flat_c = torch.empty(total, device=dev, dtype=self.cd) if self.cd != F32 else self.flat
        self.offsets = {}
        off = 0
        for name, p in named:
            n = p.numel()
            self.flat[off:off + n].copy_(p.detach().reshape(-1))
            p.data = self.flat[off:off + n].view(p.shape)
            p.grad = self.gflat[off:off + n].view(p.shape)
            self.offsets[name] = (off, n, tuple(p.shape))
            off += n
        self._refresh_compute_copy()
        self.layers = []
        self.layer_grads = []
        self.layer_slices = []
        for i, b in enumerate(model.blocks):
            names = [f"blocks.{i}.{k}" for k in ("attn_norm.weight", "attn.qkv.weight", "attn.proj.weight",
                                                   "mlp_norm.weight", "mlp.up.weight", "mlp.down.weight")]
            masters = [self.view(self.flat, n) for n in names]
            lw = engine.LayerWeights(*masters, cd=self.cd, eps_attn=b.attn_norm.eps, eps_mlp=b.mlp_norm.eps)
            lw.qkv_c, lw.proj_c, lw.up_c, lw.down_c = (self.view(self.flat_c, n) for n in names[1:3] + names[4:6])
            self.layers.append(lw)
            self.layer_grads.append(engine.LayerGrads([self.view(self.gflat, n) for n in names]))
            first, last = self.offsets[names[0]], self.offsets[names[-1]]
            self.layer_slices.append(self.gflat[first[0]:last[0] + last[1]])
        self.tok = self.view(self.flat, "token_embedding.weight")
        self.tok_c = self.view(self.flat_c, "token_embedding.weight")
        self.pos = self.view(self.flat, "position_embedding.weight")
        self.final_w = self.view(self.flat, "final_norm.weight")
        self.g_tok = self.view(self.gflat, "token_embedding.weight")
        self.g_pos = self.view(self.gflat, "position_embedding.weight")
        self.g_final = self.view(self.gflat, "final_norm.weight")
        # ---- static activation buffers
        B, T = settings.batch_size, settings.sequence_length
        if T > self.cfg.max_sequence_length:
            raise ValueError("sequence_length exceeds the model maximum")
        self.M = B * T
        V = self.cfg.vocab_size
        self.vpad = (V + 63) // 64 * 64
        self.logits = torch.empty((self.M, self.vpad), device=dev, dtype=self.cd)
        self.fused_head = settings.fused_head and self.cd in (torch.bfloat16, torch.float16)
        if self.fused_head:
            width = _lib.lib().rk_head_stats_width(V)
            self.head_stats = torch.empty((self.M, width, 2), device=dev, dtype=F32)
            self.head_xlabel = torch.empty(self.M, device=dev, dtype=F32)
            self.head_rowc = torch.empty((self.M, 4), device=dev, dtype=F32)
            self.head_fcoef = torch.empty((width, self.M), device=dev, dtype=F32)
        self.loss_rows = torch.empty(self.M, device=dev, dtype=F32)
        self.ids = torch.zeros((settings.accumulation, B, T), device=dev, dtype=torch.int64)
        self.labels = torch.full((settings.accumulation, B, T), -100, device=dev, dtype=torch.int64)
        self.inv_denominator = torch.ones((), device=dev, dtype=F32)
        self.loss_sum = torch.zeros((), device=dev, dtype=F32)
        side = torch.cuda.Stream(device=dev) if (dev.type == "cuda" and settings.overlap_wgrad) else None
        self.fwd_stream = torch.cuda.Stream(device=dev) if (dev.type == "cuda" and settings.overlap_forward) else None
        # the last microstep's rows grouped by id (the first phase of its
        # embedding backward), written on the forward stream after the later
        # forward sweeps; _sorted_m names the microstep it holds, per update
        self.emb_sorted = (torch.empty(max(_lib.lib().rk_embedding_bwd_sort_bytes(self.M, self.cfg.vocab_size), 1),
                                       device=dev, dtype=torch.uint8) if self.fwd_stream is not None else None)
        self._sorted_m = None
        self.kern = engine.LayerKernels(self.cfg.n_heads, B, T, self.cd, settings.mlp_tokens, wgrad_stream=side)
        # AdamW state (flat, fp32) and the device scalar block of rk_clip_adamw_prepare
        self.exp_avg = torch.zeros_like(self.flat)
        self.exp_avg_sq = torch.zeros_like(self.flat)
        self.opt_scalars = torch.zeros(8, device=dev, dtype=F32)
        self.opt_scalars[0] = settings.learning_rate
        self.norm_ws = torch.empty(_lib.lib().rk_clip_adamw_workspace() // 4, device=dev, dtype=F32)
        # DP buckets: one per layer (launched as the last microstep's sweep passes it),
        # then the embedding, position and final-norm gradients, the loss sum
        # (launched once the last microstep's loss is in, so every rank returns
        # the global loss) and the head's share of the tied embedding gradient.
        # Tied-gradient split (model.py:101,104; reversible.py:106): with more
        # than one rank the head weight gradients of every microstep and the
        # embedding scatters of all microsteps but the last accumulate in
        # g_head, whose bucket is launched as soon as the last head weight
        # gradient is issued, so it crosses NVLink beside the reverse sweep;
        # g_tok keeps only the last microstep's embedding scatter, and the two
        # reduced shares are summed before the optimizer.
        self.g_head = torch.zeros_like(self.g_tok) if (self.world > 1 and settings.tied_split) else None
        self.buckets = GradBuckets(self.layer_slices + [self.g_tok, self.g_pos, self.g_final, self.loss_sum]
                                   + ([self.g_head] if self.g_head is not None else []),
                                   process_group, dev) if self.world > 1 else None
        self.graph = None
        self.head_events = None

    def time_head_fprop(self):
        """Records CUDA events (graph-capturable) around each microstep's head
        GEMM from now on; head_fprop_ms() reads the durations of the last update."""
        self.head_events = [(torch.cuda.Event(enable_timing=True, external=True),
                             torch.cuda.Event(enable_timing=True, external=True))
                            for _ in range(self.s.accumulation)]

    def head_fprop_ms(self) -> list[float]:
        return [a.elapsed_time(b) for a, b in self.head_events] if self.head_events else []

    # ------------------------------------------------------------------ layout helpers
    def view(self, buf: torch.Tensor, name: str) -> torch.Tensor:
        off, n, shape = self.offsets[name]
        return buf[off:off + n].view(shape)

    def _refresh_compute_copy(self):
        if self.flat_c is not self.flat:
            self.flat_c.copy_(self.flat)

    # ------------------------------------------------------------------ data
    def stage_batches(self, batches, update_targets: int):
        """Copies this rank's microstep batches (from data.update_batches) into
        the static device buffers; the tail of a short update is padded with
        ignored targets."""
        self.ids.zero_()
        self.labels.fill_(-100)
        for m, (x, y, _) in enumerate(batches):
            self.ids[m, :x.shape[0]].copy_(x, non_blocking=True)
            self.labels[m, :y.shape[0]].copy_(y, non_blocking=True)
        self.inv_denominator.fill_(1.0 / update_targets)

    def stage_update(self, staged) -> torch.cuda.Event:
        """Copies a data.StagedUpdate (pinned ids/labels [accumulation, B, T])
        into the static device buffers with one asynchronous copy each and
        returns an event recorded after the copies (hand it to
        UpdatePrefetcher.release)."""
        if tuple(staged.ids.shape) != tuple(self.ids.shape):
            raise ValueError(f"staged batch shape {tuple(staged.ids.shape)} != {tuple(self.ids.shape)}")
        self.ids.copy_(staged.ids, non_blocking=True)
        self.labels.copy_(staged.labels, non_blocking=True)
        self.inv_denominator.fill_(1.0 / staged.update_targets)
        done = torch.cuda.Event()
        done.record()
        return done

    def train(self, prefetcher, max_updates: int | None = None, on_update=None) -> int:
        """The reference trainer's update loop (train_baseline.py:247-285) over
        a data.UpdatePrefetcher: stage the update's batches, set the
        warm-up/cosine learning rate, run the update (the captured graph when
        capture() was called). on_update(index, staged, loss_sum) sees the
        device loss sum of each update. Returns the number of updates run."""
        n = 0
        for staged in prefetcher:
            done = self.stage_update(staged)
            prefetcher.release(staged, done)
            loss = self.update(lr=learning_rate(self.s, staged.committed, staged.update_targets))
            if on_update is not None:
                on_update(n, staged, loss)
            n += 1
            if max_updates is not None and n >= max_updates:
                break
        return n

    # ------------------------------------------------------------------ checkpoints
    def _torch_adamw(self, lr: float | None = None) -> torch.optim.AdamW:
        s = self.s
        return torch.optim.AdamW(self.model.parameters(), lr=s.learning_rate if lr is None else lr,
                                 betas=(s.beta1, s.beta2), weight_decay=s.weight_decay)

    def optimizer_state_dict(self) -> dict:
        """The AdamW state in torch.optim.AdamW.state_dict() format (the
        reference checkpoint's "optimizer" entry, train_baseline.py:333): per
        parameter in model.parameters() order its step, exp_avg and exp_avg_sq."""
        opt = self._torch_adamw(float(self.opt_scalars[0]))
        step = float(self.opt_scalars[1])
        if step > 0:
            for name, p in self.model.named_parameters():
                opt.state[p] = {"step": torch.tensor(step, dtype=F32),
                                "exp_avg": self.view(self.exp_avg, name).detach().clone(),
                                "exp_avg_sq": self.view(self.exp_avg_sq, name).detach().clone()}
        return opt.state_dict()

    def load_optimizer_state_dict(self, state: dict):
        """Loads a torch.optim.AdamW state dict (the reference checkpoint's
        "optimizer" entry) into the flat moment buffers and the step count."""
        opt = self._torch_adamw()
        opt.load_state_dict(state)
        steps = set()
        for name, p in self.model.named_parameters():
            st = opt.state.get(p)
            if not st:
                self.view(self.exp_avg, name).zero_()
                self.view(self.exp_avg_sq, name).zero_()
                steps.add(0.0)
                continue
            self.view(self.exp_avg, name).copy_(st["exp_avg"])
            self.view(self.exp_avg_sq, name).copy_(st["exp_avg_sq"])
            steps.add(float(st["step"]))
        if len(steps) > 1:
            raise ValueError(f"parameters are at different AdamW steps {sorted(steps)}")
        self.opt_scalars[1] = steps.pop() if steps else 0.0
        self.opt_scalars[0] = float(opt.param_groups[0]["lr"])

    def state_dict(self) -> dict:
        """{"model", "optimizer"} as the reference checkpoint holds them
        (train_baseline.py:332-333): the module state_dict (parameter names of
        model.py) and the AdamW state."""
        return {"model": self.model.state_dict(), "optimizer": self.optimizer_state_dict()}

    def load_state_dict(self, state: dict):
        """Restores a checkpoint written by state_dict() or by the reference
        trainer (its "model" and "optimizer" entries)."""
        self.model.load_state_dict(state["model"])
        self._refresh_compute_copy()
        self.load_optimizer_state_dict(state["optimizer"])

    # ------------------------------------------------------------------ one microstep
    def _forward_states(self, m: int):
        """Microstep m's embedding and reversible forward sweep: the final (p, q)."""
        x = fn.embedding_fwd(self.ids[m], self.tok, self.pos)
        return engine.stack_forward(self.kern, self.layers, x, x, self.model.method, self.model.step_size)

    def _microstep(self, m: int, last: bool, states=None, after_head=None):
        """after_head(), if given, is called once the head GEMM is issued (the
        caller issues the next microstep's forward sweep there)."""
        cfg, s, kern = self.cfg, self.s, self.kern
        B, T, d = s.batch_size, s.sequence_length, cfg.d_model
        ids = self.ids[m]
        labels = self.labels[m].reshape(-1)
        p, q = states if states is not None else self._forward_states(m)
        # the top layer's forward recompute only needs the final states: issued
        # now, it runs beside the head
        first = kern.recompute(self.layers[-1], p, q, self.model.method, self.model.step_size) \
            if kern.pipelined(p.shape[0]) else None
        out = q if self.model.method == "midpoint" else p
        eps_f = self.model.final_norm.eps if self.model.final_norm.eps is not None else torch.finfo(F32).eps
        hidden, rstd_f = fn.rmsnorm_fwd(out, self.final_w, eps_f, out_dtype=self.cd)
        V = cfg.vocab_size
        logits = self.logits[:, :V]
        loss_rows = self.loss_rows
        if self.fused_head:
            # head GEMM with the log-sum-exp partials in its epilogue (the
            # buffer receives exp(x - block max)), per-row loss, then the two
            # backward GEMMs form dlogits = (softmax - onehot) / update_targets
            # inside the GEMM
            ev = self.head_events[m] if self.head_events is not None else None
            if ev is not None:
                ev[0].record()
            st = fn.head_fprop(hidden, self.tok_c, labels, expo=logits, stats=self.head_stats,
                               xlabel=self.head_xlabel)
            if ev is not None:
                ev[1].record()
            if after_head is not None:
                after_head()
            fn.head_loss(st, 1.0, self.inv_denominator, loss_rows=loss_rows, rowc=self.head_rowc,
                         fcoef=self.head_fcoef)
            if kern.side is not None:
                # the loss sum (and its data-parallel bucket) off the dgrad's path
                with kern.side_work():
                    self.loss_sum += loss_rows.sum()
                    loss_done = torch.cuda.Event()
                    loss_done.record()
                if last and self.world > 1:
                    self.buckets.launch(len(self.layers) + 3, after=[loss_done])
            else:
                self.loss_sum += loss_rows.sum()
                self._loss_bucket(last)
            g_head = self.g_head if self.g_head is not None else self.g_tok
            if kern.side is not None:
                # the head weight gradient runs beside the dgrad and the
                # reverse sweep; the sweep's final join (stack_backward) orders
                # it before the embedding backward, which also adds into g_tok
                with kern.side_work():
                    fn.head_wgrad(st, hidden, dw=g_head, accumulate=True)
                    head_done = torch.cuda.Event()
                    head_done.record()
                if last and self.g_head is not None:
                    self.buckets.launch(self._head_bucket, after=[head_done])
            dhidden = fn.head_dgrad(st, self.tok_c)
            if kern.side is None:
                fn.head_wgrad(st, hidden, dw=g_head, accumulate=True)
                if last and self.g_head is not None:
                    self.buckets.launch(self._head_bucket)
        else:
            fn.linear_fwd(hidden, self.tok_c, out=logits)
            if after_head is not None:
                after_head()
            # dlogits = (softmax - onehot) / update_targets, in place over the logits
            _lib.call("rk_cross_entropy_fwd_bwd", logits.data_ptr(), self.vpad, V, labels.data_ptr(), self.M, 1.0,
                      self.inv_denominator.data_ptr(), loss_rows.data_ptr(), logits.data_ptr(), self.vpad,
                      _lib.code(self.cd), -100, _lib.stream_ptr())
            self.loss_sum += loss_rows.sum()
            self._loss_bucket(last)
            dhidden = fn.linear_dgrad(logits, self.tok_c)
            fn.linear_wgrad(logits, hidden, dw=self.g_head if self.g_head is not None else self.g_tok,
                            accumulate=True)
            if last and self.g_head is not None:
                self.buckets.launch(self._head_bucket)
        # final-norm backward; its weight-gradient reduction goes to the
        # weight-gradient stream when there is one (joined by the sweep's end)
        dout, _ = kern._norm_bwd(out, self.final_w, rstd_f, dhidden, self.g_final)
        # the unused output's cotangent is zero; the engine takes None for it
        dp, dq = (None, dout) if self.model.method == "midpoint" else (dout, None)
        hook = self._bucket_hook if (last and self.world > 1) else None
        _, _, dp, dq = engine.stack_backward(kern, self.layers, self.layer_grads, p, q, dp, dq, self.model.method,
                                             self.model.step_size, on_layer_done=hook, first=first)
        # boundary p = q = embedding: both cotangents reach it (summed inside the kernel)
        # (with the tied-gradient split, earlier microsteps scatter into g_head)
        g_emb = self.g_head if (self.g_head is not None and not last) else self.g_tok
        if self._sorted_m == m:
            # the id grouping ran on the forward stream, joined before this microstep
            fn.embedding_bwd_sorted(self.emb_sorted, dp, g_emb, self.g_pos, T, dx2=dq)
        elif not last and kern.side is not None:
            # before the next microstep's head: on the weight-gradient stream,
            # ahead of that head's weight gradient (the other writer of g_tok)
            with kern.side_work():
                fn.embedding_bwd(ids, dp, g_emb, self.g_pos, dx2=dq)
            kern.hold(dp, dq)
        else:
            fn.embedding_bwd(ids, dp, g_emb, self.g_pos, dx2=dq)

    def _loss_bucket(self, last: bool):
        if last and self.world > 1:
            self.buckets.launch(len(self.layers) + 3)

    def _bucket_hook(self, layer: int, events=None):
        self.buckets.launch(layer, after=events)

    # ------------------------------------------------------------------ one update
    @property
    def _head_bucket(self) -> int:
        return len(self.layers) + 4

    def _update_body(self):
        self._sorted_m = None
        self.gflat.zero_()
        if self.g_head is not None:
            self.g_head.zero_()
        self.loss_sum.zero_()
        acc = self.s.accumulation
        if self.fwd_stream is None or acc == 1:
            for m in range(acc):
                self._microstep(m, last=(m == acc - 1))
        else:
            # Microstep m+1's forward sweep (weights are fixed within the
            # update) runs on its own stream beside microstep m's head and
            # reverse sweep; its final states stay referenced until the join.
            main = torch.cuda.current_stream()
            if self.s.forward_overlap == "start":
                # every later microstep's forward sweep beside microstep 0's
                # (the sweeps keep only their final states)
                ready = torch.cuda.Event()
                ready.record(main)
                self.fwd_stream.wait_event(ready)
                with torch.cuda.stream(self.fwd_stream):
                    later = [self._forward_states(m) for m in range(1, acc)]
                    fn.embedding_bwd_sort(self.ids[acc - 1], self.cfg.vocab_size, out=self.emb_sorted)
                    self._sorted_m = acc - 1
                done = torch.cuda.Event()
                done.record(self.fwd_stream)
                states = self._forward_states(0)
                for m in range(acc):
                    if m == 1:
                        main.wait_event(done)
                    self._microstep(m, last=(m == acc - 1), states=states)
                    states = later[m] if m + 1 < acc else None
                self._finish_update()
                return
            states = self._forward_states(0)
            for m in range(acc):
                box = {}

                def issue_next(m=m, box=box):
                    ready = torch.cuda.Event()
                    ready.record(main)
                    self.fwd_stream.wait_event(ready)
                    with torch.cuda.stream(self.fwd_stream):
                        box["states"] = self._forward_states(m + 1)
                    box["done"] = torch.cuda.Event()
                    box["done"].record(self.fwd_stream)
                later = self.s.forward_overlap == "after_head"
                if m + 1 < acc and not later:
                    issue_next()
                self._microstep(m, last=(m == acc - 1), states=states,
                                after_head=issue_next if (m + 1 < acc and later) else None)
                if "done" in box:
                    main.wait_event(box["done"])
                states = box.get("states")
        self._finish_update()

    def _finish_update(self):
        """The data-parallel exchange of the remaining buckets, then clip + AdamW."""
        if self.world > 1:
            n = len(self.layers)
            for i in range(n, n + 3):
                self.buckets.launch(i)
            self.buckets.finish()
            if self.g_head is not None:
                self.g_tok.add_(self.g_head)  # the two reduced shares of the tied gradient
        self._optimizer_step()

    def _optimizer_step(self):
        """clip_grad_norm_(max_norm) then AdamW (train_baseline.py:272,280) in two fused kernels."""
        s = self.s
        _lib.call("rk_clip_adamw_prepare", self.gflat.data_ptr(), self.gflat.numel(), float(s.grad_clip),
                  float(s.beta1), float(s.beta2), float(s.weight_decay), self.norm_ws.data_ptr(),
                  self.norm_ws.numel() * 4, self.opt_scalars.data_ptr(), _lib.stream_ptr())
        c_ptr = self.flat_c.data_ptr() if self.flat_c is not self.flat else None
        _lib.call("rk_adamw_step", self.flat.data_ptr(), self.gflat.data_ptr(), self.exp_avg.data_ptr(),
                  self.exp_avg_sq.data_ptr(), c_ptr, _lib.code(self.cd), self.flat.numel(),
                  self.opt_scalars.data_ptr(), float(s.beta1), float(s.beta2), 1e-8, _lib.stream_ptr())

    @property
    def grad_norm(self) -> torch.Tensor:
        """Pre-clip global gradient norm of the last update (device scalar)."""
        return self.opt_scalars[2]

    def update(self, lr: float | None = None):
        """Runs one update on the staged batches; returns the device loss sum.
        With capture() done, replays the CUDA graph."""
        if lr is not None:
            self.opt_scalars[0].fill_(lr)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._update_body()
        return self.loss_sum

    def capture(self, warmup: int = 1):
        """Captures one update as a CUDA graph. `warmup` eager updates run first
        (on a side stream) so every kernel's one-time host set-up is done; the
        optimizer state lives in preallocated buffers, so capture needs no
        warm-up for correctness."""
        side = torch.cuda.Stream(device=self.dev)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._update_body()
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(self.graph):
                self._update_body()
        except Exception:
            self.graph = None
            self.kern.reset_streams()
            raise
        return self.graph
