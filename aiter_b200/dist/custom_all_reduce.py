"""CustomAllreduce: the CUDA-IPC allreduce of libaiter_b200.so behind the
reference's interface (aiter/dist/device_communicators/custom_all_reduce.py:243-739).

Each rank allocates one IPC region in the library (signals + three staging buffers of
`max_size` bytes: two alternate between eager calls, one serves calls captured into
CUDA graphs); the 64-byte IPC handles are exchanged over the CPU (gloo) group,
as the reference exchanges them over its CPU group / TCP store
(custom_all_reduce.py:140-153,219-240), and every rank opens all peers' regions.
"""
import contextlib
import ctypes
import logging
from typing import Optional

import torch
import torch.distributed as dist

from .. import _lib

logger = logging.getLogger("aiter_b200")

IPC_HANDLE_BYTES = 64


def exchange_handles(group, handle: bytes):
    """All ranks' handles, in rank order, over a CPU process group."""
    world = dist.get_world_size(group=group)
    out = [None] * world
    dist.all_gather_object(out, bytes(handle), group=group)
    for h in out:
        if not isinstance(h, (bytes, bytearray)) or len(h) != IPC_HANDLE_BYTES:
            raise RuntimeError("malformed IPC handle received from a peer")
    return out


class CustomAllreduce:
    _SUPPORTED_WORLD_SIZES = [2, 4, 6, 8]

    def __init__(self, group, device, max_size=128 * 1024 * 1024, enable_register_for_capturing: bool = True):
        """`enable_register_for_capturing` is the reference's switch for reading captured
        inputs in place from registered buffers (custom_all_reduce.py:248-253); here every
        call reads its input through this rank's IPC-shared staging buffers, captured or
        not, so the flag is recorded and changes nothing."""
        self.enable_register_for_capturing = enable_register_for_capturing
        self.disabled = True
        self._IS_CAPTURING = False
        self._ctx = 0
        self.group = group
        assert dist.get_backend(group) != dist.Backend.NCCL, \
            "CustomAllreduce should be attached to a non-NCCL group."
        self.rank = dist.get_rank(group=group)
        self.world_size = dist.get_world_size(group=group)
        if self.world_size == 1:
            return
        if self.world_size not in self._SUPPORTED_WORLD_SIZES:
            logger.warning("custom allreduce disabled: unsupported world size %d", self.world_size)
            return
        if isinstance(device, int):
            device = torch.device(f"cuda:{device}")
        elif isinstance(device, str):
            device = torch.device(device)
        self.device = device
        self.max_size = int(max_size)
        L = _lib.lib()
        self._L = L
        ctx = ctypes.c_int64(0)
        handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        _lib.check_status("custom_ar_init", L.custom_ar_init(self.rank, self.world_size, self.max_size,
                                                             device.index, ctypes.byref(ctx), handle))
        self._ctx = ctx.value
        try:
            handles = exchange_handles(group, handle.raw)
            blob = b"".join(handles)
            _lib.check_status("custom_ar_open_peers", L.custom_ar_open_peers(self._ctx, blob))
        except Exception:
            L.custom_ar_dispose(self._ctx)
            self._ctx = 0
            raise
        self.disabled = False

    @contextlib.contextmanager
    def capture(self):
        """Context for CUDA-graph capture (custom_all_reduce.py:391-403 in the
        reference).  Nothing needs registering afterwards: the staging buffers are
        IPC-shared at construction, call epochs are counted on the device, and a call
        made while its stream is capturing ends with an extra barrier because every
        replay reuses the same staging buffer.  `is_capturing` mirrors the reference's
        `_IS_CAPTURING`."""
        try:
            self._IS_CAPTURING = True
            yield
        finally:
            self._IS_CAPTURING = False

    @property
    def is_capturing(self) -> bool:
        return self._IS_CAPTURING

    _DTYPES = (torch.bfloat16, torch.float16, torch.float32)

    def should_custom_ar(self, inp: torch.Tensor) -> bool:
        """Eligibility (custom_all_reduce.py:423-437): bf16, fp16 or fp32, contiguous,
        16-byte multiple, at most the registered size."""
        if self.disabled:
            return False
        nbytes = inp.numel() * inp.element_size()
        return (inp.dtype in self._DTYPES and inp.is_contiguous() and nbytes % 16 == 0
                and nbytes <= self.max_size and inp.device == self.device)

    def all_reduce(self, inp: torch.Tensor, *, out: torch.Tensor = None, two_shot=None,
                   open_fp8_quant: bool = False) -> torch.Tensor:
        """out = sum over ranks of inp, accumulated in fp32 in rank order (identical
        bits on every rank).  `open_fp8_quant` (custom_all_reduce.py:453-482): fp16
        messages of at least 128 * 2048 elements take the two-shot allreduce whose
        all-gather half moves fp8 codes with one fp16 scale per group, as the
        reference does; each rank's own segment is then exact and the others carry
        the fp8 rounding.  Other messages ignore the flag."""
        if out is None:
            out = torch.empty_like(inp)
        a, b = _lib.to_aiter(inp), _lib.to_aiter(out)
        st = _lib.current_stream_ptr(self.device.index)
        if open_fp8_quant:
            ret = self._L.custom_ar_all_reduce_fp8(self._ctx, ctypes.byref(a), ctypes.byref(b), st)
            name = "custom_ar_all_reduce_fp8"
        else:
            force = -1 if two_shot is None else (1 if two_shot else 0)
            ret = self._L.custom_ar_all_reduce(self._ctx, ctypes.byref(a), ctypes.byref(b), force, st)
            name = "custom_ar_all_reduce"
        if ret:
            _lib.check_status(name, ret)
        return out

    # ---- buffer registration (custom_all_reduce.py:405-421).  Inputs and outputs are
    # never read or written in place by peers here: each call stages through this rank's
    # IPC-shared buffers, which were exchanged at construction, so there is nothing to
    # register, eagerly or after a graph capture.
    def register_input_buffer(self, inp: torch.Tensor):
        return None

    def register_output_buffer(self, out: torch.Tensor):
        return None

    def register_graph_buffers(self):
        return None

    def _gather_last(self, inp: torch.Tensor, dim: int):
        """(eligible, along the last dim) for an all-gather of `inp` along `dim`."""
        nd = inp.dim()
        dim = dim + nd if dim < 0 else dim
        esz = inp.element_size()
        nbytes = inp.numel() * esz
        last = nd > 0 and dim == nd - 1 and dim != 0
        ok = (not self.disabled and inp.is_contiguous() and nbytes % 16 == 0
              and nbytes <= self.max_size and (dim == 0 or last)
              and not (last and (inp.shape[-1] * esz) % 16) and inp.device == self.device)
        return ok, last

    def should_custom_ag(self, inp: torch.Tensor, dim: int = 0) -> bool:
        """All-gather eligibility (custom_all_reduce.py:439-451): contiguous, a 16-byte
        multiple, this rank's input within the staging size (peers read it from there),
        along dim 0 or the last dim (the last dim also needs 16-byte rows)."""
        return self._gather_last(inp, dim)[0]

    def _allgather_out_shape(self, inp: torch.Tensor, dim: int):
        """Output shape of an all-gather along dim 0 or the last dim; 1-D otherwise
        (custom_all_reduce.py:544-553)."""
        nd = inp.dim()
        if nd == 0:
            return (self.world_size,)
        if dim == 0:
            return (inp.shape[0] * self.world_size,) + tuple(inp.shape[1:])
        if dim == -1 or dim == nd - 1:
            return tuple(inp.shape[:-1]) + (inp.shape[-1] * self.world_size,)
        return (inp.numel() * self.world_size,)

    def _all_gather(self, inp: torch.Tensor, out: Optional[torch.Tensor], dim: int) -> torch.Tensor:
        ok, last = self._gather_last(inp, dim)
        if not ok:
            raise ValueError(f"custom all-gather does not take this tensor (shape {tuple(inp.shape)}, dim {dim})")
        if out is None:
            out = torch.empty(self._allgather_out_shape(inp, dim), dtype=inp.dtype, device=inp.device)
        a, b = _lib.to_aiter(inp), _lib.to_aiter(out)
        ret = self._L.custom_ar_all_gather(self._ctx, ctypes.byref(a), ctypes.byref(b), 1 if last else 0,
                                           _lib.current_stream_ptr(self.device.index))
        if ret:
            _lib.check_status("custom_ar_all_gather", ret)
        return out

    def all_gather_reg(self, inp: torch.Tensor, out: torch.Tensor = None, dim: int = 0) -> torch.Tensor:
        """All-gather of a (captured) input (custom_all_reduce.py:555-569); the same
        staged kernel as all_gather_unreg here."""
        return self._all_gather(inp, out, dim)

    def all_gather_unreg(self, inp: torch.Tensor, out: torch.Tensor = None, dim: int = 0) -> torch.Tensor:
        """All-gather through the staging buffers (custom_all_reduce.py:571-589)."""
        return self._all_gather(inp, out, dim)

    def custom_all_gather(self, inp: torch.Tensor, dim: int = 0) -> Optional[torch.Tensor]:
        """All-gather over peer memory along dim 0 or the last dim (the reference's
        custom all-gather); None when the tensor is not eligible (size, alignment)."""
        if not self.should_custom_ag(inp, dim):
            return None
        return self._all_gather(inp, None, dim)

    def _rs_eligible(self, inp: torch.Tensor) -> bool:
        if self.disabled or inp.dtype not in self._DTYPES or not inp.is_contiguous():
            return False
        nbytes = inp.numel() * inp.element_size()
        return not (inp.numel() % self.world_size or (nbytes // self.world_size) % 16 or nbytes > self.max_size)

    def reduce_scatter(self, inp: torch.Tensor, out: torch.Tensor, *, registered: bool = False):
        """Reduce-scatter over peer memory into `out` (numel / world elements, this rank's
        share of the rank-ordered fp32 sum; custom_all_reduce.py:514-530).  `registered`
        is accepted for the reference's signature: inputs are always staged here."""
        if not self._rs_eligible(inp):
            raise ValueError(f"custom reduce-scatter does not take this tensor (shape {tuple(inp.shape)})")
        a, b = _lib.to_aiter(inp), _lib.to_aiter(out)
        ret = self._L.custom_ar_reduce_scatter(self._ctx, ctypes.byref(a), ctypes.byref(b),
                                               _lib.current_stream_ptr(self.device.index))
        if ret:
            _lib.check_status("custom_ar_reduce_scatter", ret)

    def custom_reduce_scatter(self, input: torch.Tensor, output: torch.Tensor) -> bool:
        """Reduce-scatter into `output` when the tensor is eligible (custom_all_reduce.py:
        532-542); returns whether it ran (the reference returns None either way)."""
        if not self._rs_eligible(input):
            return False
        self.reduce_scatter(input, output)
        return True

    def custom_all_reduce(self, input: torch.Tensor, use_new: bool = True, open_fp8_quant: bool = False):
        if self.disabled or not self.should_custom_ar(input):
            return None
        return self.all_reduce(input, open_fp8_quant=open_fp8_quant)

    # Largest M at which the one-kernel form is the default: on two B200s it beat the
    # two-kernel form at M <= 64, tied at 512 and lost at 2048 and above (bench.py
    # --mode gemm_ar --fused-gemm-ar).
    FUSED_MAX_M = 256

    def gemm_all_reduce(self, a: torch.Tensor, w: torch.Tensor, out: torch.Tensor = None, two_shot=None,
                        fused: bool = None):
        """allreduce(a @ w^T).  Two forms with the same result bits: the two-kernel form
        (the GEMM writes into the staging buffer and the allreduce kernel reduces it, no
        copy) and the one-kernel form (`fused=True`: the GEMM epilogue pushes its tiles
        to the peers over NVLink while the MMAs of the next tiles run, then sums them).
        `fused=None` takes the one-kernel form up to FUSED_MAX_M rows."""
        if fused is None:
            fused = a.shape[0] <= self.FUSED_MAX_M
        if out is None:
            out = torch.empty((a.shape[0], w.shape[0]), dtype=torch.bfloat16, device=a.device)
        force = -1 if two_shot is None else (1 if two_shot else 0)
        ta, tw, to = _lib.to_aiter(a), _lib.to_aiter(w), _lib.to_aiter(out)
        st = _lib.current_stream_ptr(self.device.index)
        name = "custom_ar_gemm_all_reduce_fused" if fused else "custom_ar_gemm_all_reduce"
        ret = getattr(self._L, name)(self._ctx, ctypes.byref(ta), ctypes.byref(tw), ctypes.byref(to), force, st)
        if ret:
            _lib.check_status(name, ret)
        return out

    def fused_ar_rms(self, inp: torch.Tensor, res_inp: torch.Tensor, *, res_out: torch.Tensor = None,
                     out: torch.Tensor = None, scale_out: torch.Tensor = None, w: torch.Tensor, eps: float,
                     registered: bool = False, use_1stage: bool = False, post_per_token_quant: bool = False,
                     two_shot=None):
        """allreduce(inp) + res_inp -> res_out and RMSNorm(res_out) * w -> out in one
        kernel (custom_all_reduce.py:603-660 in the reference).  With
        `post_per_token_quant` the output is fp8 with one fp32 scale per row.
        Returns (out, res_out) or (out, res_out, scale_out).  `registered` is accepted
        for the reference's signature.  The kernel is one-shot unless `two_shot` is
        True (owner ranks reduce the rows, every rank normalises them locally; same bits)
        or False/True is chosen by size with two_shot="auto"."""
        if res_out is None:
            res_out = torch.empty_like(inp)
        if post_per_token_quant:
            if out is None:
                out = torch.empty(inp.shape, dtype=torch.float8_e4m3fn, device=inp.device)
            if scale_out is None:
                scale_out = torch.empty(inp.shape[:-1] + (1,), dtype=torch.float32, device=inp.device)
        elif out is None:
            out = torch.empty_like(inp)
        ts = [_lib.to_aiter(t) for t in (inp, res_inp, res_out, out, w)]
        sc = _lib.to_aiter(scale_out) if post_per_token_quant else None
        st = _lib.current_stream_ptr(self.device.index)
        scp = ctypes.byref(sc) if sc is not None else None
        if two_shot is None or use_1stage:
            ret = self._L.custom_ar_allreduce_rmsnorm(self._ctx, *[ctypes.byref(t) for t in ts], float(eps), scp, st)
        else:
            force = -1 if two_shot == "auto" else (1 if two_shot else 0)
            ret = self._L.custom_ar_allreduce_rmsnorm_ex(self._ctx, *[ctypes.byref(t) for t in ts], float(eps), scp,
                                                         force, st)
        if ret:
            _lib.check_status("custom_ar_allreduce_rmsnorm", ret)
        return (out, res_out, scale_out) if post_per_token_quant else (out, res_out)

    def _fused_eligible(self, inp: torch.Tensor) -> bool:
        h = inp.shape[-1] if inp.dim() else 0
        return self.should_custom_ar(inp) and h % 8 == 0 and 0 < h <= 16384

    def custom_fused_ar_rms(self, input: torch.Tensor, residual_inp: torch.Tensor, weight: torch.Tensor,
                            eps: float, use_1stage: bool = False):
        if self.disabled or not self._fused_eligible(input):
            return None
        return self.fused_ar_rms(input, residual_inp, w=weight, eps=eps, use_1stage=use_1stage)

    def custom_fused_ar_rms_quant(self, input: torch.Tensor, residual_inp: torch.Tensor, weight: torch.Tensor,
                                  eps: float, use_1stage: bool = False):
        if self.disabled or not self._fused_eligible(input):
            return None
        return self.fused_ar_rms(input, residual_inp, w=weight, eps=eps, use_1stage=use_1stage,
                                 post_per_token_quant=True)

    def next_buffer_tensor(self, shape, dtype=torch.bfloat16) -> torch.Tensor:
        """A tensor viewing the staging buffer the next all_reduce will read.  A
        producer that writes its result there and passes the tensor to all_reduce
        skips the input copy.  Eagerly it is valid until the call after next; during
        a CUDA graph capture it is the buffer every captured call shares, valid until
        the next captured call."""
        ptr, nbytes = ctypes.c_int64(0), ctypes.c_int64(0)
        capturing = 1 if torch.cuda.is_current_stream_capturing() else 0
        _lib.check_status("custom_ar_next_buffer_ex",
                          _lib.lib().custom_ar_next_buffer_ex(self._ctx, capturing, ctypes.byref(ptr),
                                                              ctypes.byref(nbytes)))
        n = 1
        for d in shape:
            n *= int(d)
        esz = torch.empty((), dtype=dtype).element_size()
        if n * esz > nbytes.value:
            raise ValueError(f"{n * esz} bytes exceed the staging buffer ({nbytes.value})")
        return _lib.device_view(ptr.value, shape, dtype, self.device)

    def close(self):
        if self._ctx:
            _lib.lib().custom_ar_dispose(self._ctx)
            self._ctx = 0
        self.disabled = True

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
