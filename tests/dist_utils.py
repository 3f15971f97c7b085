"""Helpers for multi-process CPU (gloo) tests."""

from __future__ import annotations

import socket

import torch.distributed as dist


def find_free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as sock:
        sock.bind(("127.0.0.1", 0))
        return int(sock.getsockname()[1])


def init_gloo(rank: int, world: int, port: int) -> None:
    dist.init_process_group(backend="gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
