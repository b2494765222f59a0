"""Public training API on the native B200 engine.

``Trainer`` is the call a user makes: give it a config and a per-rank batch
shape, then call :meth:`Trainer.step` with token ids and targets (host or
device tensors). Under ``torchrun`` with more than one rank it runs data
parallel with the gradient communication overlapped with backward, either as
DDP (:class:`~gpt2_harness_b200.parallel.ddp_native.NativeDDP`, all-reduce,
every rank updates every parameter) or as ZeRO-2
(:class:`~gpt2_harness_b200.parallel.zero_native.NativeZeRO`, reduce-scatter,
sharded AdamW and optimiser state, fused bf16 all-gather) or as ZeRO-3
(:class:`~gpt2_harness_b200.parallel.zero3_native.NativeZeRO3`, block
parameters sharded and gathered one block ahead over NVLink).
``PipelineTrainer`` runs pipeline parallelism (GPipe or 1F1B over NCCL
point-to-point), optionally with context parallelism inside every stage.

The learning-rate schedule is the reference's (train.py:72-99): linear warmup
to ``lr`` over ``warmup_steps``, then cosine decay to ``lr * min_lr_ratio``.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist

from gpt2_harness_b200.config import GPTConfig, TrainConfig
from gpt2_harness_b200.models.engine import Engine, OptimConfig
from gpt2_harness_b200.ops import native as N

__all__ = ["Trainer", "PipelineTrainer", "lr_at_step"]


def lr_at_step(step: int, cfg: TrainConfig) -> float:
    """Warmup + cosine schedule. ``step`` counts from 0."""
    if cfg.warmup_steps > 0 and step < cfg.warmup_steps:
        return cfg.lr * (step + 1) / cfg.warmup_steps
    span = max(cfg.steps - cfg.warmup_steps, 1)
    frac = min(max((step - cfg.warmup_steps) / span, 0.0), 1.0)
    floor = cfg.lr * cfg.min_lr_ratio
    return floor + 0.5 * (cfg.lr - floor) * (1.0 + math.cos(math.pi * frac))


class Trainer:
    """GPT-2 training on native sm_100a kernels, one process per GPU.

    Args:
        config: model architecture.
        batch_size / seq_len: per-rank micro-batch shape (fixed: buffers are
            preallocated for it).
        train: optimiser settings and LR schedule (``TrainConfig``); ``None``
            uses a constant ``lr`` from its defaults.
        comm: ``"p2p"`` (fused peer-memory all-reduce), ``"mc"`` (the same
            through NVLink SHARP: multimem loads reduced in the NVSwitch) or
            ``"nccl"`` when the default process group has more than one rank
            (DDP only).
        strategy: ``"ddp"``, ``"zero2"`` or ``"zero3"`` (ignored on one rank),
            or ``"tp"``: tensor + sequence parallelism over all ranks, where
            ``batch_size`` is the GLOBAL batch every rank receives, or
            ``"cp"``: context parallelism, every rank receives the same
            ``batch_size`` full sequences of ``seq_len`` tokens and computes
            its contiguous ``seq_len / p`` slice of each.
        comm_blocks: CTAs of each fused peer-memory all-reduce that
            overlaps backward (DDP and CP, p2p).
        cp_balance: context-parallel split, ``"zigzag"`` (two chunks per rank,
            equal causal work) or ``"contiguous"`` (one slice per rank).
        cp_kv: context-parallel keys and values, ``"gather"`` (every rank
            copies the keys its queries see before attention) or ``"stream"``
            (the attention kernels read them in place from their owners).
        graph: replay the step as one CUDA graph (one rank, or native DDP).
        reduce_dtype: gradient wire of DDP and ZeRO-3, ``"fp32"`` or ``"bf16"``
            (buckets / unit reduce-scatters and root all-reduces on bf16
            copies; the P2P kernels sum in fp32).
        seed: weight init seed (identical on every rank; rank 0's weights are
            broadcast to make sure).
    """

    def __init__(self, config: GPTConfig, batch_size: int, seq_len: int, *,
                 train: Optional[TrainConfig] = None, comm: str = "p2p",
                 device: Optional[torch.device] = None, seed: int = 0,
                 bucket_bytes: int = 25 * 1024 * 1024, schedule: bool = True,
                 strategy: str = "ddp", comm_blocks: int = 128, cp_balance: str = "zigzag",
                 cp_kv: str = "gather",
                 graph: bool = False, reduce_dtype: str = "fp32") -> None:
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        torch.cuda.set_device(self.device)
        self.config = config
        self.train_cfg = train or TrainConfig()
        self.schedule = schedule and train is not None
        self.B, self.T = batch_size, seq_len
        self.world = dist.get_world_size() if dist.is_initialized() else 1
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        tc = self.train_cfg
        optim = OptimConfig(lr=tc.lr, betas=tuple(tc.betas), eps=tc.eps,
                            weight_decay=tc.weight_decay, grad_clip=tc.grad_clip)
        if strategy not in ("ddp", "zero2", "zero3", "tp", "cp"):
            raise ValueError(f"unknown strategy {strategy!r}")
        self.strategy = strategy if (self.world > 1 or strategy == "tp") else "single"
        self.cp = None
        # One CUDA graph for forward + backward (+ the DDP bucket all-reduces,
        # whose epochs come from a device counter) + optimiser update; set
        # below when allowed
        self.graph = False
        self._graph: Optional[torch.cuda.CUDAGraph] = None
        self._graph_loss: Optional[torch.Tensor] = None
        self._eager_steps = 0
        self.graph_launches = 0
        if strategy == "tp":
            # tensor + sequence parallelism: every rank takes the same global
            # batch (batch_size x seq_len) and holds 1/p of every block
            from gpt2_harness_b200.parallel.tp_native import TPEngine

            self.ddp = None
            self.engine = TPEngine(config, batch_size, seq_len, self.device, optim=optim, seed=seed)
            self.idx = torch.zeros(batch_size, seq_len, dtype=torch.int64, device=self.device)
            self.tgt = torch.zeros(batch_size, seq_len, dtype=torch.int64, device=self.device)
            self.step_num = 0
            self.h2d_done = torch.cuda.Event()
            return
        self.ddp = None
        self.cp = None
        grad_buffer = shadow_buffer = None
        if strategy == "cp" and self.world > 1:
            # context parallelism: every rank takes the same batch of full
            # sequences and computes its contiguous T/p slice of each;
            # weight gradients are averaged over the group like DDP
            from gpt2_harness_b200.models.engine import ParamLayout
            from gpt2_harness_b200.parallel.cp_native import NativeCP
            from gpt2_harness_b200.parallel.ddp_native import NativeDDP

            self.cp = NativeCP(config, batch_size, seq_len, device=self.device, balance=cp_balance, kv=cp_kv)
            self.ddp = NativeDDP(ParamLayout(config), comm=comm, bucket_bytes=bucket_bytes,
                                 device=self.device, nblocks=comm_blocks)
            grad_buffer = self.ddp.grad_buffer
            self.T_local = seq_len // self.world
        elif self.world > 1:
            from gpt2_harness_b200.models.engine import ParamLayout

            layout = ParamLayout(config)
            if strategy == "zero2":
                from gpt2_harness_b200.parallel.zero_native import NativeZeRO

                self.ddp = NativeZeRO(layout, bucket_bytes=bucket_bytes, device=self.device)
                shadow_buffer = self.ddp.shadow_buffer
            elif strategy == "zero3":
                from gpt2_harness_b200.parallel.zero3_native import NativeZeRO3

                self.ddp = NativeZeRO3(layout, device=self.device, reduce_dtype=reduce_dtype)
            else:
                from gpt2_harness_b200.parallel.ddp_native import NativeDDP

                self.ddp = NativeDDP(layout, comm=comm, bucket_bytes=bucket_bytes,
                                     device=self.device, nblocks=comm_blocks, reduce_dtype=reduce_dtype)
            grad_buffer = self.ddp.grad_buffer
        storage = self.ddp.storage_layout if self.strategy == "zero3" else None
        self.engine = Engine(config, self.device, optim=optim, grad_buffer=grad_buffer,
                             shadow_buffer=shadow_buffer, seed=seed,
                             optimizer_state=self.strategy not in ("zero2", "zero3"),
                             storage=storage)
        if self.ddp is not None:
            dist.broadcast(self.engine.master, src=0)
            self.engine.sync_shadow()
            self.ddp.attach(self.engine)
        if self.cp is not None:
            self.cp.attach(self.engine)
        self.engine.acts(batch_size, seq_len if self.cp is None else self.T_local)
        if self.cp is not None:
            self.idx_l = torch.zeros(batch_size, self.T_local, dtype=torch.int64, device=self.device)
            self.tgt_l = torch.zeros(batch_size, self.T_local, dtype=torch.int64, device=self.device)
        self.idx = torch.zeros(batch_size, seq_len, dtype=torch.int64, device=self.device)
        self.tgt = torch.zeros(batch_size, seq_len, dtype=torch.int64, device=self.device)
        self.step_num = 0
        self.h2d_done = torch.cuda.Event()
        if graph and self.ddp is not None and not (
                self.strategy == "ddp" and getattr(self.ddp, "comm", None) in ("p2p", "mc")):
            raise ValueError("graph=True replays one-rank and native-DDP steps only")
        if graph and self.ddp is not None:
            self.ddp.device_epochs = True  # before any launch
        self.graph = graph

    @property
    def num_parameters(self) -> int:
        if self.strategy == "tp":
            from gpt2_harness_b200.models.engine import ParamLayout

            return ParamLayout(self.config).num_parameters
        return self.engine.layout.num_parameters

    def _load_inputs(self, idx: torch.Tensor, targets: torch.Tensor):
        if idx.shape != (self.B, self.T) or targets.shape != (self.B, self.T):
            raise ValueError(f"expected ({self.B}, {self.T}) batches, got {tuple(idx.shape)}")
        if self.cp is not None:
            # this rank's tokens of every sequence
            self.cp.local_tokens(idx, self.idx_l)
            self.cp.local_tokens(targets, self.tgt_l)
            self.h2d_done.record()
            return self.idx_l, self.tgt_l
        if idx.device == self.device and targets.device == self.device:
            return idx, targets
        self.idx.copy_(idx, non_blocking=True)
        self.tgt.copy_(targets, non_blocking=True)
        # a caller that refills the same pinned host buffers waits on this
        # before overwriting them
        self.h2d_done.record()
        return self.idx, self.tgt

    def step_async(self, idx: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """One optimiser step; returns the loss as a device scalar (no sync).
        Host inputs should be pinned for the copy to be asynchronous."""
        eng = self.engine
        if self.schedule:
            eng.set_lr(lr_at_step(self.step_num, self.train_cfg))
        if self.graph:
            return self._graph_step(idx, targets)
        i, t = self._load_inputs(idx, targets)
        loss = eng.forward(i, t)
        if self.strategy == "tp":
            eng.backward()
        else:
            eng.backward(i)
        if self.ddp is not None:
            self.ddp.finish()
        eng.optimizer_step()
        self.step_num += 1
        return loss

    def _graph_step(self, idx: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """The step as one CUDA graph replay (one rank, or native DDP).
        Outside the graph, on the same stream: the batch is copied into the
        static input buffers and the step's AdamW scalars into the device
        buffer the update reads. The first step runs eagerly (kernel
        attributes are set, workspaces sized), the second is captured, then
        replayed every step; the kernels and their order are the eager
        step's, so the results are bit-identical."""
        eng = self.engine
        self.idx.copy_(idx, non_blocking=True)
        self.tgt.copy_(targets, non_blocking=True)
        self.h2d_done.record()
        eng.stage_hyperparams()
        if self._graph is None:
            if self._eager_steps == 0:
                self._eager_steps += 1
                loss = eng.forward(self.idx, self.tgt)
                eng.backward(self.idx)
                if self.ddp is not None:
                    self.ddp.finish()
                eng._optimizer_update()
                self.step_num += 1
                return loss
            # Ranks capture at different speeds (host work: launch encoding,
            # graph instantiation); a rank that starts replaying more than a
            # handshake's wait budget before a peer would time out its bucket
            # all-reduces and leave them out of step. Align before and after.
            torch.cuda.synchronize(self.device)
            if self.ddp is not None:
                dist.barrier(device_ids=[self.device.index])
            g = torch.cuda.CUDAGraph()
            n0 = N.lib().launch_count()
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                self._graph_loss = eng.forward(self.idx, self.tgt)
                eng.backward(self.idx)  # DDP buckets fork onto the comm stream
                if self.ddp is not None:
                    self.ddp.finish()   # ... and join back before the update
                eng._optimizer_update()
            # native kernels in the graph: each replay launches them all
            self.graph_launches = N.lib().launch_count() - n0
            if self.ddp is not None:
                dist.barrier(device_ids=[self.device.index])
            self._graph = g
        self._graph.replay()
        self.step_num += 1
        return self._graph_loss

    def step(self, idx: torch.Tensor, targets: torch.Tensor) -> float:
        """One optimiser step; returns this rank's loss as a Python float."""
        return float(self.step_async(idx, targets).item())

    def check(self) -> None:
        """Raise if any native kernel recorded an error (synchronises); a
        DDP handshake timeout names the first bucket wait that gave up."""
        try:
            N.check_errors(self.device)
        except RuntimeError as e:
            rec = self.ddp.timeout_record() if hasattr(self.ddp, "timeout_record") else None
            if rec:
                raise RuntimeError(f"{e}; first all-reduce handshake that gave up: {rec}") from e
            raise

    def state_dict(self) -> dict:
        """Model (reference names, fp32), step counters and optimiser state.
        Under ZeRO-2 the optimiser state is this rank's shard (a collective
        call: every rank must call it)."""
        if self.strategy == "tp":
            eng = self.engine
            return {"model": eng.full_state("master"), "step": self.step_num,
                    "optim_step": eng.step_count, "exp_avg": eng.full_state("exp_avg"),
                    "exp_avg_sq": eng.full_state("exp_avg_sq")}
        if self.strategy in ("zero2", "zero3"):
            eng = self.engine
            full = self.ddp.full_master()
            model = {s.name: eng.layout.view(full, s.name).clone() for s in eng.layout.specs}
            model["lm_head.weight"] = model["wte.weight"]
            return {"model": model, "step": self.step_num, "optim_step": eng.step_count,
                    "exp_avg_shard": self.ddp.exp_avg.clone(),
                    "exp_avg_sq_shard": self.ddp.exp_avg_sq.clone(), "rank": self.rank,
                    "world_size": self.world}
        return {"model": self.engine.state_dict(), "step": self.step_num,
                "exp_avg": self.engine.exp_avg.clone(), "exp_avg_sq": self.engine.exp_avg_sq.clone(),
                "optim_step": self.engine.step_count}

    def close(self) -> None:
        if self.strategy == "tp":
            self.engine.close()
            return
        self._graph = None
        if self.cp is not None:
            self.cp.close()
        if self.ddp is not None:
            self.ddp.close()


class PipelineTrainer:
    """Pipeline (x context) parallel GPT-2 training on native kernels.

    The world is a ``pp x cp`` mesh (global rank = stage * cp + c): ``pp``
    stages of ``n_layer / pp`` blocks each (stage 0 also the embeddings, the
    last stage ln_f and an untied lm_head), and within every stage ``cp``
    ranks splitting each sequence into contiguous slices (causal all-gather of
    K/V over peer memory, weight gradients averaged over the slice group).
    Every rank calls :meth:`step` with the same global batch ``[m * B, T]``
    of token ids and targets; stage 0 reads the ids, the last stage the
    targets, each of the micro-batches ``m`` rows ``[i*B, (i+1)*B)``.

    Reference semantics: src/transformer_internals/parallel/pipeline_parallel.py
    (stage split, GPipe / 1F1B, loss / m, untied head) composed with
    sequence_parallel.py (all-gather-KV attention).
    """

    def __init__(self, config: GPTConfig, micro_batch: int, seq_len: int, micro_batches: int, *,
                 pp: Optional[int] = None, cp: int = 1, schedule: str = "1f1b",
                 train: Optional[TrainConfig] = None, device: Optional[torch.device] = None,
                 seed: int = 0, comm_blocks: int = 128, cp_balance: str = "zigzag",
                 cp_kv: str = "gather") -> None:
        from gpt2_harness_b200.parallel.cp_native import NativeCP
        from gpt2_harness_b200.parallel.pp_native import StageEngine, make_mesh

        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        torch.cuda.set_device(self.device)
        if not dist.is_initialized():
            dist.init_process_group("nccl", store=dist.HashStore(), rank=0, world_size=1,
                                    device_id=self.device)
        world = dist.get_world_size()
        pp = world // cp if pp is None else pp
        if seq_len % cp:
            raise ValueError(f"seq_len={seq_len} must split evenly over cp={cp}")
        self.config, self.B, self.T, self.m = config, micro_batch, seq_len, micro_batches
        self.train_cfg = train or TrainConfig()
        self.schedule = train is not None
        tc = self.train_cfg
        optim = OptimConfig(lr=tc.lr, betas=tuple(tc.betas), eps=tc.eps,
                            weight_decay=tc.weight_decay, grad_clip=tc.grad_clip)
        self.mesh = mesh = make_mesh(pp, cp)
        self.Tl = seq_len // cp
        self.engine = StageEngine(config, micro_batch, self.Tl, micro_batches, schedule=schedule,
                                  optim=optim, group=mesh.pp_group,
                                  p2p_groups=(mesh.fwd_group, mesh.bwd_group), dp_group=mesh.cp_group,
                                  device=self.device, seed=seed, comm_blocks=comm_blocks)
        self.cp = None
        if cp > 1:
            lay = self.engine.lay
            self.cp = NativeCP(config, micro_batch, seq_len, group=mesh.cp_group, device=self.device,
                               nblocks=comm_blocks, layers=range(lay.l0, lay.l1),
                               slots=len(self.engine.slots), balance=cp_balance, kv=cp_kv)
            self.cp.attach(self.engine)
        lay = self.engine.lay
        mB = micro_batches * micro_batch
        self.idx = torch.zeros(mB, self.Tl, dtype=torch.int64, device=self.device) if lay.first else None
        self.tgt = torch.zeros(mB, self.Tl, dtype=torch.int64, device=self.device) if lay.last else None
        self.h2d_done = torch.cuda.Event()
        self.step_num = 0

    @property
    def h2d_bytes_per_step(self) -> int:
        """Bytes of inputs this rank copies to the device per step."""
        return sum(t.numel() * 8 for t in (self.idx, self.tgt) if t is not None)

    def _load(self, idx: torch.Tensor, targets: torch.Tensor):
        mB = self.m * self.B
        if idx.shape != (mB, self.T) or targets.shape != (mB, self.T):
            raise ValueError(f"expected ({mB}, {self.T}) batches, got {tuple(idx.shape)}")
        for src, dst in ((idx, self.idx), (targets, self.tgt)):
            if dst is None:
                continue
            if self.cp is not None:
                self.cp.local_tokens(src, dst)
            else:
                dst.copy_(src, non_blocking=True)
        self.h2d_done.record()
        B = self.B
        split = lambda t: [t[i * B:(i + 1) * B] for i in range(self.m)] if t is not None else [None] * self.m
        return split(self.idx), split(self.tgt)

    def step_async(self, idx: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """One optimiser step over the m micro-batches; returns the mean loss
        as a device scalar (meaningful on the last stage)."""
        if self.schedule:
            self.engine.optim.lr = lr_at_step(self.step_num, self.train_cfg)
        mi, mt = self._load(idx, targets)
        loss = self.engine.train_step(mi, mt)
        self.step_num += 1
        return loss

    def step(self, idx: torch.Tensor, targets: torch.Tensor) -> Optional[float]:
        """One optimiser step; the last stage returns its mean loss as a
        Python float, other stages ``None``."""
        loss = self.step_async(idx, targets)
        return float(loss.item()) if self.engine.lay.last else None

    def check(self) -> None:
        N.check_errors(self.device)

    def state_dict(self) -> dict:
        """This rank's stage: parameters (reference names, fp32), AdamW state,
        and where it sits in the mesh. Ranks of one CP group hold identical
        copies."""
        m = self.mesh
        return {"model": self.engine.state_dict(), "optim": self.engine.optimizer_state(),
                "step": self.step_num, "stage": m.stage, "pp": m.pp, "cp": m.cp,
                "layers": (self.engine.lay.l0, self.engine.lay.l1)}

    def load_state_dict(self, sd: dict) -> None:
        """Restore :meth:`state_dict` output of the same stage (or load a
        full-model ``{"model": ...}`` dict: only this stage's tensors are read)."""
        self.engine.load_state_dict(sd["model"], sd.get("optim"))
        self.step_num = int(sd.get("step", 0))

    def close(self) -> None:
        if self.cp is not None:
            self.cp.close()
        self.engine.close()
