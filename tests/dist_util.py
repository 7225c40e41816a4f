"""Spawn helpers for multi-process tests (127.0.0.1 rendezvous, short timeouts)."""
import os
import socket

import torch.multiprocessing as mp


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def run_ranks(fn, world, *args):
    """Run fn(rank, world, port, *args) in `world` spawned processes; re-raises."""
    port = free_port()
    mp.spawn(fn, args=(world, port) + args, nprocs=world, join=True)
