"""Multi-process CPU tests over gloo: the matched cycle at world 2 and 4,
checkpoint save / resume, the sharded-parameter runtime, and host-side failure
detection (a rank that raises, a rank that never joins).

Every rank is a spawned process with its own gloo process group on
127.0.0.1; each test bounds its own run time, so a failure can never hang the
suite.  No GPU is touched.
"""

from __future__ import annotations

import os
import socket
import time
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TINY = os.path.join(ROOT, "configs", "h3_dmd_tiny_cpu.yaml")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _env(rank: int, world: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), LOCAL_WORLD_SIZE=str(world))
    torch.set_num_threads(2)


def _run(fn, world: int, *args, timeout: float = 300.0):
    """Spawn ``world`` ranks of ``fn(rank, world, port, queue, *args)``; returns (messages, exit codes)."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, queue, *args)) for r in range(world)]
    for p in procs:
        p.start()
    deadline = time.monotonic() + timeout
    for p in procs:
        p.join(max(1.0, deadline - time.monotonic()))
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join(5)
    msgs = []
    while not queue.empty():
        msgs.append(queue.get())
    return msgs, [p.exitcode for p in procs]


def _tiny_config(world: int, out_dir: str | None = None, shard_size: int | None = None, **training):
    from h3_a100.config import load_config

    dist_cfg = {"fsdp2": {"size": shard_size or world}, "timeout_minutes": 2}
    if shard_size is not None:
        dist_cfg["hybrid_shard"] = {"enabled": True, "shard_size": shard_size}
    overrides = {
        "distributed": dist_cfg,
        "training": {"a100": {"matched_compute": {"expected_world_size": world}}, **training},
        "kernels": {"backend": "torch", "device": "cpu"},
    }
    if out_dir is not None:
        overrides["training"]["output_dir"] = out_dir
    return load_config(TINY, overrides)


# --------------------------------------------------------------------------- matched cycle at world N
def _cycle_rank(rank, world, port, queue, iters, shard_size=None):
    try:
        _env(rank, world, port)
        from h3_a100.api import build_trainer

        trainer = build_trainer(_tiny_config(world, shard_size=shard_size, max_train_iters=iters))
        trainer.setup()
        samples = trainer.samples()
        losses = [trainer.run_cycle(samples, i) for i in range(iters)]
        receipt = trainer.last_cycle_receipt
        student = trainer.model.lora["student"].flat.detach().clone()
        gathered = [torch.empty_like(student) for _ in range(world)]
        dist.all_gather(gathered, student)
        queue.put(("ok", rank, losses, receipt, all(torch.equal(gathered[0], g) for g in gathered)))
        trainer.data.close()
        dist.barrier()
    except Exception:  # noqa: BLE001 - reported to the parent
        queue.put(("error", rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world,shard_size", [(2, None), (4, None), (4, 2)], ids=["world2", "world4", "hsdp2x2"])
def test_matched_cycle_gloo(world, shard_size):
    """Full shard at world 2 and 4, and HSDP (2 replicas x 2 shards): the
    adapters stay identical on every rank of the world."""
    msgs, codes = _run(_cycle_rank, world, 2, shard_size)
    errors = [m for m in msgs if m[0] == "error"]
    assert not errors, "\n".join(m[2] for m in errors)
    assert codes == [0] * world
    oks = sorted((m for m in msgs if m[0] == "ok"), key=lambda m: m[1])
    assert len(oks) == world
    for _, _, losses, receipt, replicated in oks:
        assert replicated, "Student LoRA differs across ranks after the update"
        assert all(torch.isfinite(torch.tensor([v["dmd"], v["fake"]])).all() for v in losses)
        census = receipt["census"]
        assert census["forwards"] == {"student": 24, "fake": 6, "teacher": 1}
        assert census["backwards"] == {"student": 1, "fake": 5}
        assert census["world"] == world
        assert receipt["exact_replay"]["cache_miss_count"] == 0
        assert receipt["boundary"]["grad_checkpoint_call_count"] == 6 * 4
    # every rank drew its own samples (world x 6 unique identities, checked in-loop), so losses differ
    assert len({round(m[2][0]["fake"], 6) for m in oks}) > 1


# --------------------------------------------------------------------------- checkpoint / resume
def _resume_rank(rank, world, port, queue, out_dir):
    try:
        _env(rank, world, port)
        from h3_a100.api import build_trainer
        from h3_a100.trainer.checkpointing import find_latest_checkpoint

        # 1. train two cycles, saving after each
        t1 = build_trainer(_tiny_config(world, out_dir, max_train_iters=2, save_every_iters=1))
        t1.train()
        ref_student = t1.model.lora["student"].flat.detach().clone()
        ref_fake = t1.model.lora["fake"].flat.detach().clone()
        ref_m = t1.optimizers["fake"].exp_avg.clone()
        t1.data.close()
        dist.barrier()
        # 2. an incomplete newer checkpoint (no _SUCCESS) must be ignored
        if rank == 0:
            os.makedirs(os.path.join(out_dir, "checkpoint-000000007", "student"), exist_ok=True)
        dist.barrier()
        path, it = find_latest_checkpoint(out_dir)
        assert it == 2 and path.endswith("checkpoint-000000002"), (path, it)
        # 3. a fresh trainer resumes from it with identical adapters and optimizer state
        cfg = _tiny_config(world, out_dir, max_train_iters=2)
        cfg["resume"] = {"auto_resume": True}
        t2 = build_trainer(cfg)
        resume, current = t2._resolve_resume_a100()
        t2.setup(resume_ckpt_path=resume)
        same = (torch.equal(t2.model.lora["student"].flat, ref_student)
                and torch.equal(t2.model.lora["fake"].flat, ref_fake)
                and torch.equal(t2.optimizers["fake"].exp_avg, ref_m)
                and t2.optimizers["student"].step_count == 2 and t2.optimizers["fake"].step_count == 10)
        queue.put(("ok", rank, current, same))
        t2.data.close()
    except Exception:  # noqa: BLE001
        queue.put(("error", rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_checkpoint_resume_gloo(tmp_path):
    msgs, codes = _run(_resume_rank, 2, str(tmp_path / "out"))
    errors = [m for m in msgs if m[0] == "error"]
    assert not errors, "\n".join(m[2] for m in errors)
    assert codes == [0, 0]
    for _, _, current, same in msgs:
        assert current == 2 and same
    ckpt = tmp_path / "out" / "checkpoint-000000002"
    for name in ("_SUCCESS", "trainer_state.pt", "rank-0000.pt", "rank-0001.pt",
                 "student/pytorch_lora_weights.safetensors", "fake/pytorch_lora_weights.safetensors"):
        assert (ckpt / name).exists(), name


def _world_mismatch_rank(rank, world, port, queue, out_dir):
    try:
        _env(rank, world, port)
        from h3_a100.api import build_trainer

        cfg = _tiny_config(world, out_dir, max_train_iters=1)
        cfg["resume"] = {"auto_resume": True}
        t = build_trainer(cfg)
        try:
            resume, _ = t._resolve_resume_a100()
            t.setup(resume_ckpt_path=resume)
            queue.put(("no-error", rank))
        except RuntimeError as exc:
            queue.put(("raised", rank, str(exc)))
        t.data.close()
    except Exception:  # noqa: BLE001
        queue.put(("error", rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_resume_refuses_other_world_size(tmp_path):
    out = str(tmp_path / "out")
    msgs, _ = _run(_resume_rank, 2, out)
    assert not [m for m in msgs if m[0] == "error"]
    msgs, codes = _run(_world_mismatch_rank, 1, out)
    assert codes == [0]
    assert msgs and msgs[0][0] == "raised" and "world_size" in msgs[0][2], msgs


# --------------------------------------------------------------------------- sharded-parameter runtime
def _sharded_rank(rank, world, port, queue):
    try:
        _env(rank, world, port)
        dist.init_process_group("gloo", timeout=timedelta(seconds=60))
        from h3_a100.parallel.comm import TorchComm
        from h3_a100.parallel.sharded import ShardedUnit

        torch.manual_seed(0)   # every rank builds the same module
        mod = torch.nn.Linear(37, 19)
        ref = {k: v.detach().clone() for k, v in mod.state_dict().items()}
        comm = TorchComm(None, torch.device("cpu"))
        unit = ShardedUnit("linear", mod, ["weight", "bias"], comm)
        emptied = all(p.numel() == 0 for p in mod.parameters())
        full = unit.gather()
        restored = all(torch.equal(full[k], v) for k, v in ref.items())
        unit.release()
        queue.put(("ok", rank, emptied, restored, unit.shard.numel()))
    except Exception:  # noqa: BLE001
        queue.put(("error", rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_sharded_unit_gather_gloo():
    msgs, codes = _run(_sharded_rank, 2)
    errors = [m for m in msgs if m[0] == "error"]
    assert not errors, "\n".join(m[2] for m in errors)
    assert codes == [0, 0]
    for _, _, emptied, restored, shard in msgs:
        assert emptied and restored
        total = 37 * 19 + 19
        assert shard * 2 >= total


# --------------------------------------------------------------------------- failure detection
def _raising_rank(rank, world, port, queue):
    """Rank 1 raises between steps; rank 0's next collective must fail, not hang."""
    try:
        _env(rank, world, port)
        dist.init_process_group("gloo", timeout=timedelta(seconds=5))
        x = torch.ones(4)
        dist.all_reduce(x)          # step 1: everyone participates
        if rank == 1:
            raise RuntimeError("injected failure on rank 1")
        t0 = time.monotonic()
        try:
            dist.all_reduce(x)      # step 2: the peer is gone
            queue.put(("no-error", rank))
        except Exception as exc:  # noqa: BLE001 - gloo raises RuntimeError / DistBackendError
            queue.put(("detected", rank, time.monotonic() - t0, type(exc).__name__))
    except RuntimeError as exc:
        queue.put(("injected", rank, str(exc)))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


def test_peer_failure_is_detected_on_host():
    msgs, _ = _run(_raising_rank, 2, timeout=120)
    kinds = {m[1]: m for m in msgs}
    assert kinds[1][0] == "injected"
    assert kinds[0][0] == "detected", msgs
    assert kinds[0][2] < 60.0


def _late_rank(rank, world, port, queue):
    """Rank 1 never joins: rank 0's rendezvous ends with an error after its timeout."""
    _env(rank, world, port)
    if rank == 1:
        queue.put(("absent", rank))
        return
    t0 = time.monotonic()
    try:
        dist.init_process_group("gloo", timeout=timedelta(seconds=4))
        queue.put(("joined", rank))
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        queue.put(("detected", rank, time.monotonic() - t0, type(exc).__name__))


def test_missing_rank_times_out():
    msgs, _ = _run(_late_rank, 2, timeout=120)
    kinds = {m[1]: m for m in msgs}
    assert kinds[0][0] == "detected", msgs
    assert kinds[0][2] < 60.0
