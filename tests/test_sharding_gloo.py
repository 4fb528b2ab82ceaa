"""CPU, two gloo ranks: scene sharding, camera splitting with a gradient all-reduce,
and failure of a rank seen by the other on the host.

The renderer inside the ranks is the CPU oracle (float64), so these tests exercise
only the multi-process logic of diff_gabor_splatting_b200.sharding; the GPU kernels
are the same per rank.
"""

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from diff_gabor_splatting_b200 import sharding
from helpers import appearance_names, ordered, small_inputs

NAMES = None


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _render_loss(values, method, total_pixels):
    """Oracle render; loss = sum over this rank's pixels / all pixels of the batch."""
    from oracle import gabor_oracle as O

    rgb, alpha, meta = O.render(values["means"], values["quaternions"], values["scales"],
                                values["opacities"], [values[k] for k in appearance_names(method)],
                                values["view_matrices"], values["intrinsics"], 9, 9,
                                backgrounds=values["backgrounds"], neural=method == "neural",
                                dtype=torch.float64)
    maps = torch.cat((rgb, alpha, meta["accumulated_depth"], meta["normals"],
                      meta["distortion"]), -1)
    return (maps.square().sum()) / total_pixels


def _inputs(method, scenes, cameras):
    v = small_inputs(method, scenes=scenes, cameras=cameras, device="cpu")
    return {k: t.detach().double() for k, t in ordered(v, method).items()}


def _worker(rank, world, port, method, scenes, cameras, out_dir, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        full = _inputs(method, scenes, cameras)
        shards = sharding.plan(scenes, cameras, world)
        groups = sharding.groups_for(shards)
        shard = shards[rank]
        mine = {k: t.clone().requires_grad_() for k, t in sharding.take(full, shard).items()}
        total = scenes * cameras * 81
        if rank == fail_rank:
            raise RuntimeError("injected failure before the gradient all-reduce")
        _render_loss(mine, method, total).backward()
        if shard.split:
            params = [t for k, t in mine.items() if k not in sharding.PER_CAMERA]
            sharding.allreduce_gradients(params, groups[shard.group_ranks])
        torch.save({k: t.grad for k, t in mine.items()}, os.path.join(out_dir, f"grads{rank}.pt"))
    except RuntimeError as error:
        with open(os.path.join(out_dir, f"error{rank}.txt"), "w") as f:
            f.write(str(error))
        raise
    finally:
        dist.destroy_process_group()


def _run(tmp_path, method, scenes, cameras, world=2, fail_rank=-1):
    port = _free_port()
    ctx = mp.start_processes(_worker, args=(world, port, method, scenes, cameras, str(tmp_path),
                                            fail_rank),
                             nprocs=world, start_method="spawn", join=False)
    while not ctx.join(timeout=60):
        pass


def test_plan_covers_every_image_once():
    for scenes, cameras, world in [(32, 8, 1), (32, 8, 2), (32, 8, 8), (8, 16, 4), (1, 4, 2),
                                   (1, 4, 4), (2, 16, 8)]:
        seen = {}
        for rank, shard in enumerate(sharding.plan(scenes, cameras, world)):
            for s in range(scenes)[shard.scenes]:
                for c in range(cameras)[shard.cameras]:
                    assert (s, c) not in seen
                    seen[(s, c)] = rank
            assert rank in shard.group_ranks
        assert len(seen) == scenes * cameras
    with pytest.raises(ValueError):
        sharding.plan(1, 2, 4)   # more ranks per scene than cameras


@pytest.mark.parametrize("method", ["classic", "neural"])
def test_camera_split_allreduce_equals_single_process(tmp_path, method):
    _run(tmp_path, method, scenes=1, cameras=2)
    full = {k: t.clone().requires_grad_() for k, t in _inputs(method, 1, 2).items()}
    _render_loss(full, method, 2 * 81).backward()
    for rank in range(2):
        grads = torch.load(tmp_path / f"grads{rank}.pt")
        shard = sharding.plan(1, 2, 2)[rank]
        for name, g in grads.items():
            expected = full[name].grad[shard.scenes]
            if name in sharding.PER_CAMERA:
                expected = expected[:, shard.cameras]
            torch.testing.assert_close(g, expected, rtol=1e-9, atol=1e-12, msg=name)


def test_scene_sharding_needs_no_collective(tmp_path):
    _run(tmp_path, "classic", scenes=2, cameras=2)
    full = {k: t.clone().requires_grad_() for k, t in _inputs("classic", 2, 2).items()}
    _render_loss(full, "classic", 4 * 81).backward()
    for rank in range(2):
        grads = torch.load(tmp_path / f"grads{rank}.pt")
        for name, g in grads.items():
            torch.testing.assert_close(g, full[name].grad[rank:rank + 1], rtol=1e-9, atol=1e-12)


def test_failed_rank_is_seen_by_its_peer(tmp_path):
    """Rank 1 fails before the gradient all-reduce; rank 0's collective ends with an
    error (gloo sees the peer gone, or the short process-group timeout expires)
    instead of waiting for ever."""
    with pytest.raises(Exception):
        _run(tmp_path, "classic", scenes=1, cameras=2, fail_rank=1)
    assert (tmp_path / "error1.txt").read_text().startswith("injected failure")
    assert not (tmp_path / "grads0.pt").exists()
