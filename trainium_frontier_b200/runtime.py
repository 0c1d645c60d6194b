"""Process / device runtime: one process per GPU, NCCL over NVLink for the plumbing.

Same public surface as the reference's runtime layer (``train.py:1345-1401``,
``prepare.py:81-93``): ``detect_device_type``, ``init_runtime``, ``cleanup_runtime``,
``synchronize``, ``compute_dtype_for``, ``get_dist_info``, ``print0``.  Differences
are B200-specific: the process group gets a bounded timeout (so a rank that dies
ends its peers' next collective with an error instead of a hang), and the CUDA
device is bound before the group is created so NCCL can use it eagerly.
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def get_dist_info() -> tuple[bool, int, int, int]:
    if all(k in os.environ for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE")):
        return True, int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"]), int(os.environ["WORLD_SIZE"])
    return False, 0, 0, 1


def print0(*args, **kwargs) -> None:
    if int(os.environ.get("RANK", "0")) == 0:
        print(*args, **kwargs)


def detect_device_type(requested: str = "") -> str:
    if requested:
        return requested
    return "cuda" if torch.cuda.is_available() else "cpu"


def init_runtime(device_type: str, seed: int = 42, timeout_s: float | None = None):
    """Returns ``(ddp, rank, local_rank, world_size, device)`` like the reference."""
    assert device_type in {"cpu", "cuda"}
    torch.manual_seed(seed)
    ddp, rank, local_rank, world_size = get_dist_info()
    if timeout_s is None:
        timeout_s = float(os.environ.get("TFB200_PG_TIMEOUT_S", "600"))
    timeout = datetime.timedelta(seconds=timeout_s)
    if ddp and device_type == "cuda":
        device = torch.device("cuda", local_rank)
        torch.cuda.set_device(device)
        if not dist.is_initialized():
            dist.init_process_group("nccl", device_id=device, timeout=timeout)
    elif ddp:
        if not dist.is_initialized():
            dist.init_process_group("gloo", timeout=timeout)
        device = torch.device("cpu")
    else:
        device = torch.device(device_type)
        if device_type == "cuda":
            torch.cuda.set_device(device)
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
    return ddp, rank, local_rank, world_size, device


def cleanup_runtime() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()


def synchronize(device: torch.device) -> None:
    if device.type == "cuda":
        torch.cuda.synchronize(device)


def compute_dtype_for(device: torch.device) -> torch.dtype:
    """bf16 on the GPU, fp32 on the CPU (the CPU path is the numerical oracle)."""
    return torch.bfloat16 if device.type == "cuda" else torch.float32


def is_dist() -> bool:
    return dist.is_available() and dist.is_initialized()


def world() -> tuple[int, int]:
    if is_dist():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1
