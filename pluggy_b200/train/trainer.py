"""Training orchestrator (JSON config -> model, mesh, parallelism, optimizer, data, loop).

Parity: reference ``pluggy/train/trainer.py:62-538``:

* phases: build -> init -> parallelize -> re-seed -> objective -> optimizer ->
  scheduler -> dataloader -> checkpointer -> resume -> wandb -> prefetcher;
* same seed on every rank for build/init, then ``seed + 1 + dp_coord``;
* grad accumulation ``K = global_batch / (micro * dp)``; ``train_step`` runs
  K-1 microbatches with ``requires_sync=False`` and the last with ``True``,
  then ``sync`` -> clip -> ``optimizer.step`` -> ``zero_grad`` ->
  ``scheduler.step`` -> dp-average of the loss;
* checkpoint layout/resume rules (mesh and data sources must be unchanged);
* the rank-0 step line ``step=.. || loss=.. || gnorm=.. || lr=.. || tps=..``
  (byte-compatible: the web UI scrapes it) and ``peak cuda mem``;
* optional wandb on rank 0, asserted on every rank first.

B200 differences:

* no torch.compile and no autocast: on CUDA the models run their fused
  sm_100a sublayers in bf16 with fp32 master weights and an fp32 residual;
* the grad-norm clip coefficient stays on the device and is folded into the
  fused AdamW kernel (no extra pass over the grads, no host sync);
* the loop also runs on CPU (gloo) for the plumbing config and the tests;
* ``data.synthetic`` selects the offline Zipf token source (no tokenizer);
* ``parallelism`` accepts ``ddp`` / ``fsdp2`` plus mesh axes ``tp`` (tensor +
  sequence parallel) and ``ep`` (expert parallel); FSDP2 checkpoints are
  written sharded with placement metadata.
"""

from __future__ import annotations

import json
import os
import warnings
from datetime import datetime

import torch
import torch.nn as nn

from pluggy_b200.checkpoint.checkpointer import Checkpointer
from pluggy_b200.train.failure import FailureNotice
from pluggy_b200.core.collective import all_reduce, barrier
from pluggy_b200.core.grad_helper import clip_grad_norm
from pluggy_b200.core.mesh import Mesh
from pluggy_b200.dataloader.prefetcher import CUDAPrefetcher
from pluggy_b200.models.builder import build_model
from pluggy_b200.objectives.builder import build_objective
from pluggy_b200.optimizer.builder import build_optimizer, build_scheduler
from pluggy_b200.utils import debug_time, get_project_dir, record_time

try:
    import wandb

    HAS_WANDB = True
except ImportError:  # pragma: no cover
    HAS_WANDB = False


def load_json(path: str) -> dict:
    with open(path) as f:
        return json.load(f)


class Trainer:
    def __init__(self, train_config_path: str | dict, rank: int, local_rank: int, world_size: int,
                 benchmark: bool = False, checkpoint_root: str | None = None):
        self.config = load_json(train_config_path) if isinstance(train_config_path, str) else \
            dict(train_config_path)
        from pluggy_b200.train.validate import validate_config

        validate_config(self.config)
        self.rank, self.world_size, self.benchmark = rank, world_size, benchmark
        if torch.cuda.is_available():
            torch.cuda.set_device(local_rank)
            self.device = torch.device("cuda", local_rank)
        else:
            self.device = torch.device("cpu")
        self.mesh = Mesh(self.config["mesh"])
        self.dp_size = self.mesh.size("dp")
        self.ignore_index = self.config["objective"]["config"].get("ignore_index", -100)
        data_cfg = self.config["data"]
        self.tokenizer = None
        if not data_cfg.get("synthetic"):
            from tokenizers import Tokenizer

            self.tokenizer = Tokenizer.from_pretrained(data_cfg["tokenizer"])
        self.seed = self.config.get("seed", 0)
        torch.manual_seed(self.seed)

        self.model = self._build_model()
        self._init_weights(self.model)
        self.model = self._parallelize(self.model)
        torch.manual_seed(self.seed + 1 + self.mesh.coordinate("dp"))

        self.objective = build_objective(self.config["objective"]["name"],
                                         self.config["objective"]["config"])
        opt = self.config["optimizer"]
        self.optimizer = build_optimizer(self.model, opt["name"], opt["config"])
        if self.parallelism == "ddp":
            # ZeRO-1 data parallelism updates this rank's slices only
            self.optimizer = self.dp.zero1_optimizer(self.optimizer)
        # the optimizer writes the bf16 copies the GEMMs read (no per-step recast);
        # FSDP2 gathers full weights per step, so there is nothing to keep current
        wc = getattr(self.model, "weight_cache", None)
        if (wc is not None and self.parallelism == "ddp"
                and hasattr(self.optimizer, "add_shadow_listener")):
            wc.bind_optimizer(self.optimizer)
        self.scheduler = build_scheduler(self.optimizer, opt["scheduler"])
        self.num_train_steps = opt["scheduler"]["total_steps"]
        self.max_norm = opt.get("max_norm")

        self.dataloader = self._build_dataloader()
        self.global_batch_size = data_cfg["global_batch_size"]
        self.micro_batch_size = data_cfg["micro_batch_size"]
        per_backward = self.micro_batch_size * self.dp_size
        assert self.global_batch_size % per_backward == 0, (
            f"global_batch_size {self.global_batch_size} must be divisible by micro_batch_size "
            f"{self.micro_batch_size} x dp {self.dp_size} = {per_backward}")
        self.microbatches_per_step = self.global_batch_size // per_backward

        stamp = datetime.now().strftime("%Y-%m-%d_%H-%M-%S")
        self.run_name = f"{self.config['run_name']}_{stamp}"
        root = checkpoint_root or os.path.join(get_project_dir(), "checkpoints")
        self.checkpointer = Checkpointer(os.path.join(root, self.config["run_name"]))
        ck = self.config.get("checkpointing", {})
        self.resume = ck.get("resume")
        self.save_steps = ck.get("save_steps", 10**9)
        self.resume_scheduler = ck.get("resume_scheduler", True)
        self.resume_wandb_id = None
        # how often (optimizer steps) the kernels' status word is read; 0 = never
        self.status_check_steps = int(self.config.get("status_check_steps", 1))
        # "cuda_graph": true replays the whole step (forward, loss, backward, clip, AdamW)
        # from one CUDA graph after an eager first step (single GPU, plain data parallelism)
        self.cuda_graph = bool(self.config.get("cuda_graph", False))
        self._graph = None
        self._graph_eager_steps = 1
        # a rank that fails tells the others through the process group's store; each
        # rank checks before every step ("failure_notice": false turns it off)
        self.failure_notice = FailureNotice(rank, enabled=bool(self.config.get("failure_notice", True)))
        self.start_step = self._resume()
        self._setup_wandb()
        # the synthetic source generates batches on the host: do it on a worker thread
        background = self.device.type == "cuda" and bool(self.config["data"].get("synthetic"))
        self.prefetcher = CUDAPrefetcher(self.dataloader, self.device, background=background)

    # ---------------------------------------------------------------- building
    def _build_model(self) -> nn.Module:
        m = self.config["model"]
        return build_model(m["name"], m["config"])

    def _init_weights(self, model: nn.Module) -> None:
        model.to(self.device)
        model.init_weights()
        init_from = self.config["model"].get("init_from_hf")
        if init_from:
            from pluggy_b200.models.hf_import import load_hf_weights, weight_files

            if self.rank == 0:
                weight_files(init_from)
            if self.world_size > 1:
                barrier()
            n = load_hf_weights(model, init_from)
            if self.rank == 0:
                print(f"init_from_hf: loaded {n} tensors from {init_from}")

    def _parallelize(self, model: nn.Module) -> nn.Module:
        self.parallelism = self.config.get("parallelism", "ddp")
        sizes = self.config["mesh"]
        self.tp = None
        if sizes.get("tp", 1) > 1:
            from pluggy_b200.parallel.tensor_parallel import parallelize_tp

            tp_cfg = self.config.get("tp", {})
            self.tp = parallelize_tp(model, self.mesh, "tp",
                                     sequence_parallel=tp_cfg.get("sequence_parallel", True),
                                     fused=tp_cfg.get("fused"))
        self.cp = None
        if sizes.get("cp", 1) > 1:
            from pluggy_b200.parallel.context_parallel import parallelize_cp

            self.cp = parallelize_cp(model, self.mesh, "cp")
        # expert parallelism: "ep": {"dim": axis} splits the experts over that mesh
        # axis (normally the dp axis itself: EP = DP)
        self.ep = None
        ep_cfg = self.config.get("ep")
        if ep_cfg:
            from pluggy_b200.parallel.expert_parallel import parallelize_ep

            self.ep_dim = ep_cfg.get("dim", "dp") if isinstance(ep_cfg, dict) else "dp"
            if self.mesh.size(self.ep_dim) > 1:
                self.ep = parallelize_ep(model, self.mesh, self.ep_dim)
        if self.parallelism == "ddp":
            from pluggy_b200.parallel.ddp import DDP

            ddp_cfg = self.config.get("ddp", {})
            reducer = ddp_cfg.get("reducer", "auto")
            # ZeRO-1 leaves only each rank's slice of the gradients averaged and sums the
            # clip's squares during the reduce-scatter: it composes with plain data
            # parallelism only (tensor/context parallelism reduce more axes afterwards,
            # expert parameters are not bucketed)
            plain = self.tp is None and self.cp is None and self.ep is None
            adamw = self.config["optimizer"].get("name") == "adamw"
            if reducer == "auto":
                reducer = "zero1" if (self.device.type == "cuda" and plain and adamw
                                      and self.dp_size > 1) else "nccl"
            elif reducer == "zero1" and not (plain and adamw):
                raise ValueError("ddp.reducer 'zero1' composes with plain data parallelism and AdamW "
                                 "only (no tp, cp or ep axes); use 'fused' or 'nccl'")
            self.dp = DDP(model, self.mesh, dim="dp", bucket_mb=ddp_cfg.get("bucket_mb", 25),
                          reducer=reducer)
        elif self.parallelism == "fsdp2":
            from pluggy_b200.parallel.fsdp2 import FSDP2

            fs_cfg = self.config.get("fsdp2", {})
            self.dp = FSDP2(model, self.mesh, dim="dp", gather=fs_cfg.get("gather", "auto"),
                            lowp_gather=fs_cfg.get("lowp_gather", True),
                            reduce=fs_cfg.get("reduce", "nccl"))
        else:
            raise ValueError(f"unknown parallelism {self.parallelism!r}: expected 'ddp' or 'fsdp2'")
        self.grad_shard_dims = ("dp",) if (self.parallelism == "fsdp2" and self.dp_size > 1) else ()
        return model

    def _build_dataloader(self):
        data = self.config["data"]
        if data.get("synthetic"):
            from pluggy_b200.dataloader.builder import build_synthetic_loader

            vocab = self.config["model"]["config"]["vocab_size"]
            return build_synthetic_loader(data, vocab, self.mesh.coordinate("dp"),
                                          pin=self.device.type == "cuda")
        from pluggy_b200.dataloader.builder import build_dataloader

        return build_dataloader(data, self.tokenizer, self.ignore_index, self.mesh.coordinate("dp"),
                                self.mesh.size("dp"))

    # ------------------------------------------------------------------- wandb
    def _setup_wandb(self) -> None:
        self.wandb_run = None
        cfg = self.config.get("wandb", {})
        if not cfg.get("enabled", False) or self.benchmark:
            return
        assert HAS_WANDB, "wandb.enabled is true in the config but wandb isn't installed"
        if self.rank != 0:
            return
        self.wandb_run = wandb.init(project=cfg.get("project", "pluggy"), entity=cfg.get("entity"),
                                    name=self.run_name, id=self.resume_wandb_id,
                                    resume="must" if self.resume_wandb_id else None,
                                    config=self.config)

    def _log_metrics(self, metrics, step, tokens_per_step, t) -> None:
        jsonl = self.config.get("logging", {}).get("jsonl")
        if self.wandb_run is None and not jsonl:
            return
        log = {"train/loss": float(metrics["loss"]), "train/grad_norm": float(metrics["grad_norm"]),
               "train/lr": self.scheduler.get_last_lr()[0], "train/tokens": step * tokens_per_step,
               "perf/tps": tokens_per_step / t, "perf/step_time": t}
        if self.device.type == "cuda":
            log["perf/peak_mem_gib"] = torch.cuda.max_memory_allocated() / 2**30
        counts = getattr(self.model, "last_tokens_per_expert", None)
        if isinstance(counts, torch.Tensor) and counts.numel():
            # tokens routed to each expert (summed over the sparse layers) this step
            c = counts.detach().float().reshape(-1, counts.shape[-1]).sum(0)
            log["moe/expert_load_max_over_mean"] = float(c.max() / c.mean().clamp_min(1e-9))
        if self.wandb_run is not None:
            self.wandb_run.log(log, step=step)
        if jsonl:
            # one JSON object per optimizer step (rank 0), appended: survives restarts
            with open(jsonl, "a") as f:
                f.write(json.dumps({"step": step, **log}) + "\n")

    # -------------------------------------------------------------- checkpoint
    def _model_sharded(self) -> bool:
        """Tensor or expert parallelism: ranks hold different parameter shards."""
        return getattr(self, "tp", None) is not None or getattr(self, "ep", None) is not None

    def _full_model_state(self) -> dict[str, torch.Tensor]:
        """The unsharded model state (collective when TP/EP shard the params)."""
        sd = {k: v for k, v in self.model.state_dict().items()}
        for handle in (getattr(self, "tp", None), getattr(self, "ep", None)):
            if handle is not None:
                full = handle.full_state_dict()
                sd.update({k: full[k] for k in sd if full[k].shape != sd[k].shape})
        return sd

    def _load_full_model_state(self, sd: dict[str, torch.Tensor]) -> None:
        local = {}
        for name, t in self.model.state_dict().items():
            full = sd[name]
            mod_name = name.rpartition(".")[0]
            mod = self.model.get_submodule(mod_name) if mod_name else self.model
            if full.shape != t.shape:
                first = getattr(mod, "first", None)
                if first is not None:  # expert shard
                    full = full[first:first + t.shape[0]]
                else:  # tensor-parallel shard along the dimension that shrank
                    d = 0 if full.shape[0] != t.shape[0] else 1
                    r = self.mesh.coordinate("tp")
                    k = t.shape[d]
                    full = full.narrow(d, r * k, k)
            local[name] = full
        self.model.load_state_dict(local)

    def check_device_status(self) -> None:
        """Raise if a bounded wait in one of this rank's kernels gave up since the
        last check (a peer that never answered, a stalled pipeline stage). Such a
        kernel returns early and leaves its outputs incomplete, so training must
        not go on from them, nor checkpoint them. One int32 read per call."""
        if self.device.type != "cuda":
            return
        from pluggy_b200.ops import _ext

        if _ext.available():
            _ext.check_status(self.device)

    def _optimizer_sharded(self) -> bool:
        """ZeRO-1 data parallelism: each rank holds the AdamW state of its slices only."""
        return getattr(getattr(self, "dp", None), "zero1", None) is not None

    def checkpoint(self, step: int) -> None:
        self.check_device_status()
        if hasattr(self.optimizer, "wait_params"):
            self.optimizer.wait_params()
        if self._optimizer_sharded():
            if self.rank == 0:
                self.checkpointer.save_model(self.model, step)
            torch.save(self.optimizer.state_dict(),
                       os.path.join(self.checkpointer._step_dir(step, True),
                                    f"optimizer_rank{self.rank}.pt"))
        elif self.parallelism == "fsdp2" and self.dp_size > 1:
            self._checkpoint_sharded(step)
        elif self._model_sharded():
            sd = self._full_model_state()
            if self.rank == 0:
                torch.save(sd, self.checkpointer._path(step, "model.pt", create=True))
            torch.save(self.optimizer.state_dict(),
                       os.path.join(self.checkpointer._step_dir(step, True),
                                    f"optimizer_rank{self.rank}.pt"))
        elif self.rank == 0:
            self.checkpointer.save_model(self.model, step)
        if self.rank == 0:
            if not (self.parallelism == "fsdp2" and self.dp_size > 1) and not self._model_sharded() \
                    and not self._optimizer_sharded():
                self.checkpointer.save_optimizer(self.optimizer, step)
            self.checkpointer.save_scheduler(self.scheduler, step)
            self.checkpointer.save_trainer({"step": step, "config": self.config,
                                            "wandb_id": self.wandb_run.id if self.wandb_run else None},
                                           step)
        rng = {"cpu_rng": torch.get_rng_state()}
        if self.device.type == "cuda":
            rng["cuda_rng"] = torch.cuda.get_rng_state(self.device)
        self.checkpointer.save_rng(rng, step, self.rank)
        self.checkpointer.save_dataloader_state(self.prefetcher.loader_state_dict(), step,
                                                self.mesh.coordinate("dp"))
        barrier()
        if self.rank == 0:
            self.checkpointer.mark_complete(step)

    def _checkpoint_sharded(self, step: int) -> None:
        coord, n = self.mesh.coordinate("dp"), self.dp_size
        local = {k: v for k, v in self.model.state_dict().items()}
        placements = {k: {"dim": 0, "coord": coord, "axis_size": n} for k in local}
        self.checkpointer.save_sharded_model(local, placements, step, self.rank, self.world_size)
        torch.save(self.optimizer.state_dict(),
                   os.path.join(self.checkpointer._step_dir(step, True), f"optimizer_rank{self.rank}.pt"))

    def _resume(self) -> int:
        if self.resume is None:
            return 0
        if self.resume == "auto":
            step = self.checkpointer.latest()
            if step is None:
                return 0
        elif isinstance(self.resume, int):
            step = self.checkpointer.valid_step(self.resume)
            assert step is not None, "non valid step to resume from"
        else:
            raise ValueError("resume must be None, 'auto', or a completed training step")
        state = self.checkpointer.load_trainer(step)
        assert state["config"]["mesh"] == self.config["mesh"], (
            f"resume across a mesh change is unsupported: checkpoint has {state['config']['mesh']}, "
            f"config has {self.config['mesh']}")
        from pluggy_b200.dataloader.builder import resolve_sources

        def ids(cfg):
            if cfg["data"].get("synthetic"):
                return [("synthetic", json.dumps(cfg["data"]["synthetic"], sort_keys=True))]
            return [(s["label"], s["config"], s["split"]) for s in resolve_sources(cfg["data"])]

        assert ids(state["config"]) == ids(self.config), (
            f"resume across a change of data sources is unsupported: checkpoint has "
            f"{ids(state['config'])}, config has {ids(self.config)}")
        if self.parallelism == "fsdp2" and self.dp_size > 1:
            shard = self.checkpointer._load(step, f"model_shard_rank{self.rank}.pt")
            self.model.load_state_dict(shard)
            self.optimizer.load_state_dict(self.checkpointer._load(step, f"optimizer_rank{self.rank}.pt"))
        elif self._model_sharded():
            self._load_full_model_state(self.checkpointer._load(step, "model.pt"))
            self.optimizer.load_state_dict(self.checkpointer._load(step, f"optimizer_rank{self.rank}.pt"))
        elif self._optimizer_sharded():
            self.checkpointer.load_model(self.model, step)
            self.optimizer.load_state_dict(self.checkpointer._load(step, f"optimizer_rank{self.rank}.pt"))
        else:
            self.checkpointer.load_model(self.model, step)
            self.checkpointer.load_optimizer(self.optimizer, step)
        if self.resume_scheduler:
            self.checkpointer.load_scheduler(self.scheduler, step)
        else:
            self.scheduler.last_epoch = step
        self.checkpointer.load_dataloader(self.dataloader, step, self.mesh.coordinate("dp"))
        rng = self.checkpointer.load_rng(step, self.rank)
        if rng is None:
            rng = {k: state[k] for k in ("cpu_rng", "cuda_rng") if k in state}
        if "cpu_rng" in rng:
            torch.set_rng_state(rng["cpu_rng"])
        if "cuda_rng" in rng and self.device.type == "cuda":
            torch.cuda.set_rng_state(rng["cuda_rng"], self.device)
        self.resume_wandb_id = state.get("wandb_id")
        return state["step"]

    # -------------------------------------------------------------------- loop
    def get_batch_prefetcher(self):
        return next(self.prefetcher)

    def micro_train_step(self, batch=None) -> torch.Tensor:
        batch = self.get_batch_prefetcher() if batch is None else batch
        loss = self.objective.compute_loss(self.model, batch) / self.microbatches_per_step
        loss.backward()
        return loss.detach()

    def optimizer_step(self, scheduler_step: bool = True) -> torch.Tensor:
        """sync -> clip -> step -> zero_grad -> scheduler; returns the grad norm."""
        if self.tp is not None:
            self.tp.sync_replicated_grads()
        self.dp.sync()
        if self.cp is not None:
            self.cp.sync_grads()
        partial = []
        if self.ep is not None:
            self.ep.finish_grads(average_over_dim=self.ep_dim == "dp")
            partial.append(((self.ep_dim,), self.ep.expert_param_ids()))
        if self.tp is not None:
            ids = self.tp.sharded_param_ids()
            if self.ep is not None:
                ids = ids - self.ep.expert_param_ids()
            partial.append((("tp",), ids))
        partial = partial or None
        fused = self.device.type == "cuda" and hasattr(self.optimizer, "set_grad_scale")
        # the fused DDP reducer already summed the squares of the averaged grads
        pre = None
        if partial is None and not self.grad_shard_dims and hasattr(self.dp, "reduced_norm_sq"):
            pre = self.dp.reduced_norm_sq()
        if fused:
            gnorm, coef = clip_grad_norm(self.model.parameters(), self.mesh, self.max_norm,
                                         shard_dims=self.grad_shard_dims, fold_into_optimizer=True,
                                         partial_over=partial, precomputed_sq=pre)
            self.optimizer.set_grad_scale(coef)
        else:
            gnorm = clip_grad_norm(self.model.parameters(), self.mesh, self.max_norm,
                                   shard_dims=self.grad_shard_dims, partial_over=partial)
        self.optimizer.step()
        self.optimizer.zero_grad()
        if scheduler_step:
            self.scheduler.step()
        return gnorm

    # ------------------------------------------------------------ CUDA graph
    def _graph_ok(self) -> str | None:
        if self.device.type != "cuda":
            return "needs a CUDA device"
        if self.world_size != 1 or any(x is not None for x in (self.tp, self.cp, self.ep)):
            return "runs on one GPU without tp, cp or ep"
        if self.microbatches_per_step != 1:
            return "needs one microbatch per step"
        if not (hasattr(self.optimizer, "use_device_hyper") and self.optimizer.use_kernel):
            return "needs the fused AdamW optimizer"
        return None

    def _graph_step(self) -> dict[str, torch.Tensor]:
        """One step replayed from a CUDA graph. The first call runs eagerly (lazy state,
        kernel attributes, tensor maps); the second captures the step on the batch
        buffers it then refills before every replay. The host keeps what the graph
        cannot: the step count, the learning rate and the bias corrections (uploaded
        to the optimizer's device hyperparameters) and the scheduler."""
        batch = self.get_batch_prefetcher()
        if self._graph is None and self._graph_eager_steps > 0:
            self._graph_eager_steps -= 1
            loss = self.micro_train_step(batch)
            return {"loss": loss, "grad_norm": self.optimizer_step()}
        if self._graph is None:
            why = self._graph_ok()
            if why is not None:
                raise ValueError(f"cuda_graph {why}")
            self._static_batch = {k: v.clone() for k, v in batch.items()}
            torch.cuda.synchronize(self.device)
            torch.cuda.empty_cache()  # the graph's pool takes the eager step's cached blocks
            from pluggy_b200.utils.launch_count import count_launches

            g = torch.cuda.CUDAGraph()
            try:
                self.optimizer.use_device_hyper(self.device)
                with count_launches() as cnt, torch.cuda.graph(g):
                    loss = self.micro_train_step(self._static_batch)
                    gnorm = self.optimizer_step(scheduler_step=False)
            except (RuntimeError, AssertionError) as e:
                # nothing of the captured step ran: continue with eager steps
                warnings.warn(f"cuda_graph: capture failed, running eager steps ({e})")
                self.cuda_graph, self.optimizer._hyper = False, None
                self.optimizer.zero_grad()
                loss = self.micro_train_step(batch)
                return {"loss": loss, "grad_norm": self.optimizer_step()}
            self._graph, self._static_out = g, (loss, gnorm)
            self.graph_kernels = cnt.count  # this package's kernels in one replay
        else:
            for k, v in batch.items():
                self._static_batch[k].copy_(v, non_blocking=True)
        self.optimizer.advance()
        self._graph.replay()
        self.scheduler.step()
        loss, gnorm = self._static_out
        return {"loss": loss.clone(), "grad_norm": gnorm.clone()}

    def _train_step(self) -> dict[str, torch.Tensor]:
        if self.cuda_graph:
            return self._graph_step()
        loss = torch.zeros((), device=self.device)
        self.dp.requires_sync = False
        for _ in range(self.microbatches_per_step - 1):
            loss += self.micro_train_step()
        self.dp.requires_sync = True
        loss += self.micro_train_step()
        gnorm = self.optimizer_step()
        if self.dp_size > 1:
            all_reduce(loss, self.mesh, "dp", "avg")
        return {"loss": loss, "grad_norm": gnorm}

    train_step = record_time(_train_step)

    def _line(self, step, metrics, tokens_per_step, t) -> str:
        return (f"step={step} || loss={metrics['loss']:.4f} || gnorm={metrics['grad_norm']:.3f} "
                f"|| lr={self.scheduler.get_last_lr()[0]:.2e} || tps={tokens_per_step / t:.0f}")

    @debug_time
    def train_n_step_test(self, n_steps: int) -> None:
        tokens_per_step = self.config["data"]["seq_len"] * self.global_batch_size
        try:
            for step in range(n_steps):
                self.failure_notice.check()
                metrics, t = self.train_step()
                if self.status_check_steps and (step + 1) % self.status_check_steps == 0:
                    self.check_device_status()
                if self.rank == 0:
                    print(self._line(step, metrics, tokens_per_step, t))
        except BaseException as e:
            self.failure_notice.announce(e)
            raise
        self._print_peak()

    def _print_peak(self) -> None:
        if self.rank == 0 and self.device.type == "cuda":
            print(f"peak cuda mem: {torch.cuda.max_memory_allocated() / 2**30:.2f} GiB")

    def train(self) -> None:
        tokens_per_step = self.config["data"]["seq_len"] * self.global_batch_size
        try:
            for step in range(self.start_step, self.num_train_steps):
                self.failure_notice.check()
                metrics, t = self.train_step()
                if self.status_check_steps and (step + 1) % self.status_check_steps == 0:
                    self.check_device_status()
                if ((step + 1) % self.save_steps == 0 and step != 0) or (step + 1) == self.num_train_steps:
                    self.checkpoint(step + 1)
                if self.rank == 0:
                    self._log_metrics(metrics, step + 1, tokens_per_step, t)
                    print(self._line(step, metrics, tokens_per_step, t))
            self._print_peak()
        except BaseException as e:
            self.failure_notice.announce(e)
            raise
        finally:
            if self.wandb_run is not None:
                self.wandb_run.finish()
