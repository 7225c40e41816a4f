"""Expert-parallel dispatch / combine over NVLink (libaiter_b200.so), behind the
interface of MoRI's EpDispatchCombineOp as the reference uses it
(op_tests/multigpu_tests/test_dispatch_combine.py:110-171) and of the reference's
all2all manager (aiter/dist/device_communicators/all2all.py:21-98).

    cfg = EpDispatchCombineConfig(data_type=torch.float8_e4m3fn, rank=r, world_size=W,
                                  hidden_dim=D, scale_dim=D // 128, scale_type_size=4,
                                  max_token_type_size=2, max_num_inp_token_per_rank=T_max,
                                  num_experts_per_rank=E // W, num_experts_per_token=k)
    op = EpDispatchCombineOp(cfg)
    x, w, s, ids, n = op.dispatch(tokens_fp8, topk_weights, scales, topk_ids)
    y = aiter_b200.fused_moe(x, w1_local, w2_local, w, ids, expert_mask,
                             num_local_tokens=n, a1_scale=s, ...)
    out = op.combine(y, topk_weights, topk_ids)        # [T, D], this rank's tokens

Single node only (the reference's InterNodeV1 kernels are not built): intra-node
traffic goes over CUDA IPC peer memory.  The received rows are ordered by source
rank, then token; `combine` sums each token's outputs over the ranks it went to in
rank order in fp32.  dispatch and combine must alternate.  The MoRI launch knobs
(block_num, warp_per_block, kernel_type, rdma_block_num, gpu_per_node) are accepted
and ignored.
"""
import ctypes
import dataclasses
from typing import Optional

import torch
import torch.distributed as dist

from .. import _lib

IPC_HANDLE_BYTES = 64
_dtype_code = _lib.dtype_code


@dataclasses.dataclass
class EpDispatchCombineConfig:
    data_type: torch.dtype
    rank: int
    world_size: int
    hidden_dim: int
    scale_dim: int
    scale_type_size: int
    max_token_type_size: int
    max_num_inp_token_per_rank: int
    num_experts_per_rank: int
    num_experts_per_token: int
    warp_num_per_block: int = 16
    block_num: int = 80
    kernel_type: object = None
    rdma_block_num: int = 0
    gpu_per_node: int = 8
    # dtype of the expert outputs combine() sums (bf16 or fp16); not a MoRI field
    out_dtype: torch.dtype = torch.bfloat16


def _check_config(cfg: EpDispatchCombineConfig):
    if cfg.data_type not in (torch.float8_e4m3fn, torch.bfloat16, torch.float16):
        raise ValueError(f"unsupported token dtype {cfg.data_type}")
    if cfg.scale_dim > 0 and cfg.scale_type_size != 4:
        raise ValueError("scales must be float32 (scale_type_size 4)")
    if cfg.out_dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("out_dtype must be bf16 or fp16")
    if not 2 <= cfg.world_size <= 8:
        raise ValueError("world_size must be in [2, 8]")


class EpDispatchCombineOp:
    """One rank's dispatch / combine communicator.  Collective to construct: every
    rank of `group` (a CPU / gloo group; default: a new gloo group over WORLD)
    builds one with the same configuration."""

    def __init__(self, config: EpDispatchCombineConfig, group=None, device: Optional[torch.device] = None):
        _check_config(config)
        self.config = config
        self._ctx = 0
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        if group is None:
            group = dist.new_group(backend="gloo")
        self.group = group
        L = _lib.lib()
        self._L = L
        ctx = ctypes.c_int64(0)
        handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        _lib.check_status("ep_init", L.ep_init(
            config.rank, config.world_size, config.hidden_dim, _dtype_code(config.data_type),
            max(0, config.scale_dim), config.max_num_inp_token_per_rank, config.num_experts_per_rank,
            config.num_experts_per_token, _dtype_code(config.out_dtype), self.device.index, ctypes.byref(ctx), handle))
        self._ctx = ctx.value
        try:
            handles = [None] * config.world_size
            dist.all_gather_object(handles, handle.raw, group=group)
            if any(not isinstance(h, (bytes, bytearray)) or len(h) != IPC_HANDLE_BYTES for h in handles):
                raise RuntimeError("malformed IPC handle received from a peer")
            _lib.check_status("ep_open_handles", L.ep_open_handles(self._ctx, b"".join(handles)))
            self._views = self._make_views(lambda ptrs, rows: L.ep_buffers(self._ctx, ptrs, rows))
        except Exception:
            L.ep_destroy(self._ctx)
            self._ctx = 0
            raise

    def _make_views(self, query):
        cfg = self.config
        ptrs = (ctypes.c_int64 * 6)()
        rows = ctypes.c_int64(0)
        _lib.check_status("ep_buffers", query(ptrs, ctypes.byref(rows)))
        n = rows.value
        dv = lambda i, shape, dt: _lib.device_view(ptrs[i], shape, dt, self.device)
        k = cfg.num_experts_per_token
        return {
            "tokens": dv(0, (n, cfg.hidden_dim), cfg.data_type),
            "scales": dv(1, (n, cfg.scale_dim), torch.float32) if cfg.scale_dim > 0 else None,
            "ids": dv(2, (n, k), torch.int32),
            "weights": dv(3, (n, k), torch.float32),
            "recv_num": dv(4, (1,), torch.int32),
            "src": dv(5, (n,), torch.int32),
        }

    @property
    def capacity(self) -> int:
        return self.config.world_size * self.config.max_num_inp_token_per_rank

    def dispatch(self, input: torch.Tensor, weights: torch.Tensor, scales: Optional[torch.Tensor],
                 indices: torch.Tensor, block_num: int = -1, warp_per_block: int = -1):
        """Returns (tokens, weights, scales, ids, recv_num): views of this rank's
        receive arrays ([world * max_tokens, ...] rows, the first recv_num valid) and
        the received count as a device int32 tensor of one element."""
        ta = [_lib.to_aiter(t.contiguous()) for t in (input, weights.to(torch.float32), indices.to(torch.int32))]
        sc = _lib.to_aiter(scales.to(torch.float32).contiguous()) if scales is not None else None
        st = _lib.current_stream_ptr(self.device.index)
        ret = self._L.ep_dispatch(self._ctx, ctypes.byref(ta[0]), ctypes.byref(ta[1]),
                                  ctypes.byref(sc) if sc is not None else None, ctypes.byref(ta[2]), st)
        if ret:
            _lib.check_status("ep_dispatch", ret)
        v = self._views
        return v["tokens"], v["weights"], v["scales"], v["ids"], v["recv_num"]

    def combine(self, input: torch.Tensor, weights: Optional[torch.Tensor] = None,
                indices: Optional[torch.Tensor] = None, block_num: int = -1, warp_per_block: int = -1,
                call_reset: bool = False) -> torch.Tensor:
        """input: the expert outputs of the received rows ([world * max_tokens,
        hidden], row i for received row i).  Returns [T, hidden] for this rank's T
        tokens of the last dispatch.  weights / indices are accepted for MoRI's
        signature; the outputs are summed as they are (the MoE applied the weights)."""
        T = self._last_tokens(indices)
        y = torch.empty((T, self.config.hidden_dim), dtype=self.config.out_dtype, device=self.device)
        a, b = _lib.to_aiter(input), _lib.to_aiter(y)
        ret = self._L.ep_combine(self._ctx, ctypes.byref(a), ctypes.byref(b), _lib.current_stream_ptr(self.device.index))
        if ret:
            _lib.check_status("ep_combine", ret)
        return y

    def _last_tokens(self, indices):
        if indices is None:
            raise ValueError("combine needs the dispatch's indices to size its output")
        return int(indices.shape[0])

    def get_dispatch_src_token_pos(self) -> torch.Tensor:
        """Source position (source rank * max_tokens + token) of every received row
        of the last dispatch (synchronises to read the count)."""
        n = int(self._views["recv_num"].item())
        tags = self._views["src"][:n].to(torch.int64)
        return (tags >> 24) * self.config.max_num_inp_token_per_rank + (tags & 0xFFFFFF)

    def close(self):
        if self._ctx:
            self._L.ep_destroy(self._ctx)
            self._ctx = 0

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


class EpAll2AllManager:
    """The role of the reference's MoriAll2AllManager (all2all.py:21-98): builds and
    caches one EpDispatchCombineOp per configuration (`get_handle(kwargs)` with the
    keyword arguments of `_make_all2all_kwargs`)."""

    def __init__(self, cpu_group):
        self.cpu_group = cpu_group
        self.rank = dist.get_rank(cpu_group)
        self.world_size = dist.get_world_size(cpu_group)
        self.internode = False
        self._cache = {}

    def _make_all2all_kwargs(self, rank, num_ep_ranks, input_dtype, quant_dtype, token_hidden_size, scale_dim,
                             scale_type_size, max_num_tokens_per_dp_rank, num_local_experts, num_experts_per_token,
                             gpu_per_node=8):
        return dict(rank=rank, world_size=num_ep_ranks, data_type=quant_dtype, hidden_dim=token_hidden_size,
                    scale_dim=scale_dim, scale_type_size=scale_type_size,
                    max_token_type_size=input_dtype.itemsize, max_num_inp_token_per_rank=max_num_tokens_per_dp_rank,
                    num_experts_per_rank=num_local_experts, num_experts_per_token=num_experts_per_token,
                    gpu_per_node=gpu_per_node)

    def get_handle(self, kwargs) -> EpDispatchCombineOp:
        cfg_kwargs = self._make_all2all_kwargs(**kwargs)
        key = tuple(sorted((k, str(v)) for k, v in cfg_kwargs.items()))
        op = self._cache.get(key)
        if op is None:
            op = EpDispatchCombineOp(EpDispatchCombineConfig(**cfg_kwargs), group=self.cpu_group)
            self._cache[key] = op
        return op

    def destroy(self):
        for op in self._cache.values():
            op.close()
        self._cache.clear()


def emulated_dispatch_combine(tokens, weights, scales, ids, experts_per_rank, expert_fn, out_dtype=torch.bfloat16,
                              max_tokens=None):
    """Test hook: dispatch -> expert_fn -> combine for world = tokens.shape[0] ranks
    emulated on one GPU (ep_emu_*).  tokens [W, T, H]; expert_fn(rank, recv_tokens,
    recv_scales, recv_ids, recv_weights, n) returns [W * max_tokens, H] outputs.
    Returns (y [W, T, H], per-rank received views)."""
    L = _lib.lib()
    W, T, H = tokens.shape
    k = ids.shape[-1]
    max_tokens = T if max_tokens is None else max_tokens
    sd = scales.shape[-1] if scales is not None else 0
    dev = tokens.device
    ctx = ctypes.c_int64(0)
    _lib.check_status("ep_emu_init", L.ep_emu_init(W, H, _dtype_code(tokens.dtype), sd, max_tokens, experts_per_rank,
                                                   k, _dtype_code(out_dtype), dev.index, ctypes.byref(ctx)))
    try:
        ta = [_lib.to_aiter(t.contiguous()) for t in (tokens, weights, ids)]
        sc = _lib.to_aiter(scales.contiguous()) if scales is not None else None
        st = _lib.current_stream_ptr(dev.index)
        _lib.check_status("ep_emu_dispatch", L.ep_emu_dispatch(ctx.value, ctypes.byref(ta[0]), ctypes.byref(ta[1]),
                                                               ctypes.byref(sc) if sc is not None else None,
                                                               ctypes.byref(ta[2]), st))
        recv = []
        outs = []
        for r in range(W):
            ptrs = (ctypes.c_int64 * 6)()
            rows = ctypes.c_int64(0)
            _lib.check_status("ep_emu_buffers", L.ep_emu_buffers(ctx.value, r, ptrs, ctypes.byref(rows)))
            n_rows = rows.value
            dv = lambda i, shape, dt: _lib.device_view(ptrs[i], shape, dt, dev)
            v = {"tokens": dv(0, (n_rows, H), tokens.dtype), "scales": dv(1, (n_rows, sd), torch.float32) if sd else None,
                 "ids": dv(2, (n_rows, k), torch.int32), "weights": dv(3, (n_rows, k), torch.float32),
                 "recv_num": dv(4, (1,), torch.int32), "src": dv(5, (n_rows,), torch.int32)}
            n = int(v["recv_num"].item())
            recv.append({key: (val[:n].clone() if val is not None and key != "recv_num" else val)
                         for key, val in v.items()})
            recv[-1]["recv_num"] = n
            outs.append(expert_fn(r, v["tokens"], v["scales"], v["ids"], v["weights"], n))
        out = torch.stack(outs).to(out_dtype).contiguous()
        y = torch.empty((W, T, H), dtype=out_dtype, device=dev)
        a, b = _lib.to_aiter(out), _lib.to_aiter(y)
        _lib.check_status("ep_emu_combine", L.ep_emu_combine(ctx.value, ctypes.byref(a), ctypes.byref(b),
                                                             _lib.current_stream_ptr(dev.index)))
        return y, recv
    finally:
        L.ep_destroy(ctx.value)
