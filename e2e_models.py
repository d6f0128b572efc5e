"""End-to-end training steps whose residual paths are CGHC hyper-connections.

Two synthetic workloads with random init and seeded synthetic data (the
reference ships no such models and no datasets reach this machine):

* ``vit``: a 32x32 RGB image classifier, patch 4 (64 tokens), D = 384,
  6 blocks, 6 heads, MLP 4x, 10 classes, global batch 512 images;
* ``lm``: a decoder-only language model, 12 blocks, D = 2048, 16 heads,
  MLP 4x, vocabulary 32,000, sequence 2048, global batch 64 sequences.

Every block has two sublayers (attention, MLP), each wrapped by
``hyperconnections_b200.cghc.ContinuousGenHyperConnections`` with n = 4
streams and m = 1 (the reference layer's defaults otherwise:
conservative + PSD dissipation, no projection): the residual state is
[batch, tokens, 4 * D] in bf16, the embedding is copied into the four streams
and the streams are summed before the final norm. A training step is
forward + backward of the cross-entropy loss under bf16 autocast (fp32 master
weights) and one fused AdamW update. Under torch.distributed the global batch
is split evenly over the ranks (strong scaling), the model is wrapped in
DistributedDataParallel (NCCL gradient all-reduce in buckets overlapped with
the backward), and a rank's share is processed in micro-batches with
gradient accumulation (all but the last under ``no_sync``).
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from hyperconnections_b200.cghc import ContinuousGenHyperConnections

N_STREAMS = 4


@dataclass(frozen=True)
class Spec:
    name: str
    dim: int
    depth: int
    heads: int
    global_batch: int       # images or sequences per optimizer step, all ranks together
    seq: int                # tokens per sample
    micro_batch: int        # samples per forward/backward on one rank
    classes: int = 10       # vit
    vocab: int = 32000      # lm
    patch: int = 4          # vit


VIT = Spec("vit", dim=384, depth=6, heads=6, global_batch=512, seq=64, micro_batch=512)
LM = Spec("lm", dim=2048, depth=12, heads=16, global_batch=64, seq=2048, micro_batch=8)


class Attention(nn.Module):
    def __init__(self, dim: int, heads: int, causal: bool):
        super().__init__()
        self.norm = nn.LayerNorm(dim)
        self.qkv = nn.Linear(dim, 3 * dim)
        self.out = nn.Linear(dim, dim)
        self.heads, self.causal = heads, causal

    def forward(self, x):
        B, S, D = x.shape
        q, k, v = self.qkv(self.norm(x)).view(B, S, 3, self.heads, D // self.heads).permute(2, 0, 3, 1, 4)
        y = F.scaled_dot_product_attention(q, k, v, is_causal=self.causal)
        return self.out(y.transpose(1, 2).reshape(B, S, D))


class MLP(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.norm = nn.LayerNorm(dim)
        self.fc1 = nn.Linear(dim, 4 * dim)
        self.fc2 = nn.Linear(4 * dim, dim)

    def forward(self, x):
        return self.fc2(F.gelu(self.fc1(self.norm(x)), approximate="tanh"))


def hc(dim: int, module: nn.Module) -> ContinuousGenHyperConnections:
    return ContinuousGenHyperConnections(N_STREAMS, 1, N_STREAMS * dim, dim, module)


class Backbone(nn.Module):
    """Blocks of CGHC-wrapped attention and MLP over n bf16 streams."""

    def __init__(self, spec: Spec, causal: bool):
        super().__init__()
        self.layers = nn.ModuleList()
        for _ in range(spec.depth):
            self.layers.append(hc(spec.dim, Attention(spec.dim, spec.heads, causal)))
            self.layers.append(hc(spec.dim, MLP(spec.dim)))
        self.norm = nn.LayerNorm(spec.dim)

    def forward(self, h):
        x = h.to(torch.bfloat16).repeat(1, 1, N_STREAMS)  # the embedding in every stream
        for layer in self.layers:
            x = layer(x)
        B, S, _ = x.shape
        return self.norm(x.view(B, S, N_STREAMS, -1).sum(2))


class VisionTransformer(nn.Module):
    def __init__(self, spec: Spec = VIT):
        super().__init__()
        self.patch = nn.Conv2d(3, spec.dim, spec.patch, spec.patch)
        self.pos = nn.Parameter(0.02 * torch.randn(1, spec.seq, spec.dim))
        self.body = Backbone(spec, causal=False)
        self.head = nn.Linear(spec.dim, spec.classes)

    def forward(self, images, labels):
        h = self.patch(images).flatten(2).transpose(1, 2) + self.pos
        logits = self.head(self.body(h).mean(1))
        return F.cross_entropy(logits.float(), labels)


class DecoderLM(nn.Module):
    def __init__(self, spec: Spec = LM):
        super().__init__()
        self.embed = nn.Embedding(spec.vocab, spec.dim)
        self.pos = nn.Parameter(0.02 * torch.randn(1, spec.seq, spec.dim))
        self.body = Backbone(spec, causal=True)
        self.head = nn.Linear(spec.dim, spec.vocab, bias=False)

    def forward(self, ids, targets):
        h = self.embed(ids) + self.pos[:, : ids.shape[1]]
        logits = self.head(self.body(h))
        return F.cross_entropy(logits.float().flatten(0, 1), targets.flatten())


def build(spec: Spec):
    return VisionTransformer(spec) if spec.name == "vit" else DecoderLM(spec)


def batch(spec: Spec, samples: int, seed: int):
    """Seeded synthetic inputs on the CPU: images ~ N(0,1) with labels uniform
    in [0, 10), or token ids uniform in [0, vocab) with next-token targets."""
    g = torch.Generator().manual_seed(seed)
    if spec.name == "vit":
        return (torch.randn(samples, 3, 32, 32, generator=g), torch.randint(0, spec.classes, (samples,), generator=g))
    ids = torch.randint(0, spec.vocab, (samples, spec.seq + 1), generator=g)
    return ids[:, :-1].contiguous(), ids[:, 1:].contiguous()


class Trainer:
    """One rank's share of the training step (see module doc)."""

    def __init__(self, spec: Spec, device, world: int = 1, rank: int = 0, micro_batch: int | None = None,
                 seed: int = 0, model_fn=None):
        if spec.global_batch % world:
            raise ValueError(f"global batch {spec.global_batch} does not split over {world} ranks")
        self.spec, self.device, self.world = spec, device, world
        torch.manual_seed(seed)  # identical initial weights on every rank
        model = (model_fn or build)(spec).to(device)
        self.params = sum(p.numel() for p in model.parameters())
        self.grad_bytes = sum(p.numel() * p.element_size() for p in model.parameters() if p.requires_grad)
        if world > 1:
            ids = [device.index] if device.type == "cuda" else None
            model = nn.parallel.DistributedDataParallel(model, device_ids=ids, gradient_as_bucket_view=True)
        self.model = model
        fused = device.type == "cuda"
        self.opt = torch.optim.AdamW(model.parameters(), lr=1e-4, weight_decay=0.01, fused=fused)
        self.local_batch = spec.global_batch // world
        mb = min(micro_batch or spec.micro_batch, self.local_batch)
        while self.local_batch % mb:
            mb -= 1
        self.micro_batch = mb
        inputs, targets = batch(spec, self.local_batch, seed=1000 + rank)
        self.inputs = inputs.to(device)
        self.targets = targets.to(device)
        self.amp = device.type == "cuda"

    @property
    def tokens_per_step(self) -> int:
        return self.spec.global_batch * self.spec.seq

    def step(self, sync: bool = True) -> torch.Tensor:
        """One optimizer step over this rank's share; sync=False keeps every
        micro-batch under no_sync (no gradient all-reduce: a measurement of
        the compute alone, which leaves the replicas' weights diverging)."""
        self.opt.zero_grad(set_to_none=True)
        n_micro = self.local_batch // self.micro_batch
        total = torch.zeros((), device=self.device)
        for i in range(n_micro):
            sl = slice(i * self.micro_batch, (i + 1) * self.micro_batch)
            last = i == n_micro - 1
            ctx = self.model.no_sync() if (self.world > 1 and not (last and sync)) else _null()
            with ctx:
                with torch.autocast(self.device.type, dtype=torch.bfloat16, enabled=self.amp):
                    loss = self.model(self.inputs[sl], self.targets[sl]) / n_micro
                loss.backward()
            total += loss.detach()
        self.opt.step()
        return total


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def time_steps(trainer: Trainer, steps: int, warmup: int, sync: bool = True, barrier=None):
    """Device time (ms) of each of `steps` optimizer steps after `warmup`
    untimed ones, CUDA events on the current stream; also the last loss."""
    dev = trainer.device
    for _ in range(warmup):
        trainer.step(sync)
    torch.cuda.synchronize(dev)
    if barrier:
        barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    t0 = time.perf_counter()
    loss = None
    for e0, e1 in evs:
        e0.record()
        loss = trainer.step(sync)
        e1.record()
    torch.cuda.synchronize(dev)
    if barrier:
        barrier()
    wall = (t0, time.perf_counter())
    return [a.elapsed_time(b) for a, b in evs], float(loss.item()), wall


def time_allreduce(nbytes: int, device, world: int, reps: int = 5) -> float:
    """Device ms of one NCCL all-reduce of `nbytes` of fp32 (the gradient
    volume of one step), mean of `reps` after one warm-up."""
    buf = torch.ones(max(1, nbytes // 4), dtype=torch.float32, device=device)
    torch.distributed.all_reduce(buf)
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        torch.distributed.all_reduce(buf)
    e1.record()
    torch.cuda.synchronize(device)
    del buf
    return e0.elapsed_time(e1) / reps


def flops_per_token(spec: Spec) -> float:
    """Dense training FLOPs per token (6 per weight of the blocks and head,
    plus the attention score / value products), for context only."""
    D, L = spec.dim, spec.depth
    block = 12 * D * D
    head = D * (spec.vocab if spec.name == "lm" else 0)
    attn = 2 * 2 * spec.seq * D * (0.5 if spec.name == "lm" else 1.0)
    return 6 * (L * block + head) + 3 * L * attn


def describe(spec: Spec) -> dict:
    return {"model": spec.name, "dim": spec.dim, "depth": spec.depth, "heads": spec.heads,
            "global_batch": spec.global_batch, "seq_len": spec.seq, "hc_streams": N_STREAMS,
            "tokens_per_step": spec.global_batch * spec.seq, "mlp": "4x", "dtype": "bf16 autocast, fp32 master weights",
            **({"vocab": spec.vocab} if spec.name == "lm" else {"patch": spec.patch, "classes": spec.classes,
                                                               "image": "32x32x3"})}


def sanity(spec: Spec) -> float:
    """log(classes or vocab): the loss of a uniform prediction."""
    return math.log(spec.classes if spec.name == "vit" else spec.vocab)
