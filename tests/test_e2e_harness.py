"""Host logic of the end-to-end training harness (e2e_models.Trainer) on CPU
ranks (gloo, world size 2), with a small CPU model standing in for the
CUDA-backed ViT / LM: the global batch splits evenly over the ranks, a rank's
share runs in micro-batches with gradient accumulation, DDP all-reduces the
gradients once per step so the replicas stay identical, and a step with
every micro-batch under no_sync leaves them diverging (the measurement of the
compute alone). The synthetic data and the specs are checked on one rank."""

import os
import socket
import sys
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import e2e_models as em  # noqa: E402

TINY = em.Spec("vit", dim=8, depth=1, heads=2, global_batch=12, seq=64, micro_batch=2)


class TinyClassifier(nn.Module):
    def __init__(self, spec):
        super().__init__()
        self.fc = nn.Linear(3 * 32 * 32, spec.classes)

    def forward(self, images, labels):
        return F.cross_entropy(self.fc(images.flatten(1)), labels)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        tr = em.Trainer(TINY, torch.device("cpu"), world, rank, model_fn=TinyClassifier)
        w0 = tr.model.module.fc.weight.detach().clone()
        tr.step(sync=True)
        synced = tr.model.module.fc.weight.detach().clone()
        tr.step(sync=False)
        unsynced = tr.model.module.fc.weight.detach().clone()
        gathered = [torch.zeros_like(synced) for _ in range(world)]
        dist.all_gather(gathered, synced)
        gathered_u = [torch.zeros_like(unsynced) for _ in range(world)]
        dist.all_gather(gathered_u, unsynced)
        q.put((rank, tr.local_batch, tr.micro_batch, bool(torch.equal(gathered[0], gathered[1])),
               bool(torch.equal(gathered_u[0], gathered_u[1])), bool(torch.equal(w0, synced)),
               tr.inputs[0, 0, 0, :4].tolist()))
    finally:
        dist.destroy_process_group()


def test_ddp_micro_batches_and_sync():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, local, micro, same_synced, same_unsynced, unchanged, head in res:
        assert local == TINY.global_batch // world == 6
        assert micro == 2  # 3 micro-batches with gradient accumulation
        assert same_synced, "DDP-synchronised step left the replicas different"
        assert not same_unsynced, "a no_sync step must not all-reduce"
        assert not unchanged
    assert res[0][-1] != res[1][-1], "every rank draws its own share of the batch"


def test_specs_and_batches():
    assert em.VIT.seq == (32 // em.VIT.patch) ** 2 == 64
    assert em.LM.global_batch * em.LM.seq == 131072
    ids, tgt = em.batch(em.LM, 2, seed=0)
    assert ids.shape == (2, 2048) and torch.equal(ids[:, 1:], tgt[:, :-1])
    assert 0 <= int(ids.min()) and int(ids.max()) < em.LM.vocab
    img, lab = em.batch(em.VIT, 5, seed=0)
    assert img.shape == (5, 3, 32, 32) and lab.shape == (5,) and int(lab.max()) < 10
    d = em.describe(em.LM)
    assert d["hc_streams"] == 4 and d["tokens_per_step"] == 131072
