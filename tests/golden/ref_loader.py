"""Load the reference's own pure-torch functions from a reference checkout by AST
extraction (fixture generation only; needs the checkout, never runs on the GPU box).

`import aiter` fails without ROCm (aiter/jit/utils/cpp_extension.py:94), and the
op_tests modules run sweeps at import time, so the function definitions are
parsed out of the source files and executed in a namespace that provides the few
names they use (torch, dtypes, the enums, `get_torch_act`).  Nothing from the
reference is copied into this repository: the functions are read from the
checkout each time `make_golden.py` runs.
"""
import ast
import enum
import functools
import sys
import types

import torch
import torch.nn.functional as F


class ActivationType(enum.Enum):
    No = -1
    Silu = 0
    Gelu = 1
    Swiglu = 2


class QuantType(enum.IntEnum):
    No = 0
    per_Tensor = 1
    per_Token = 2
    per_1x32 = 3
    per_1x128 = 4
    per_128x128 = 5
    per_256x128 = 6
    per_1024x128 = 7


def _dtypes_ns():
    d = types.SimpleNamespace()
    d.fp8 = torch.float8_e4m3fn
    d.fp8_e8m0 = torch.float8_e8m0fnu
    d.fp4x2 = torch.float4_e2m1fn_x2
    d.fp16, d.bf16, d.fp32 = torch.float16, torch.bfloat16, torch.float32
    d.i32, d.i8, d.u32 = torch.int32, torch.int8, torch.uint32
    return d


def _get_torch_act(a):
    return {ActivationType.No: lambda *x, **k: x[0], ActivationType.Silu: F.silu,
            ActivationType.Gelu: F.gelu}.get(a)


def _extract(path, names, nested_in=None):
    src = open(path).read()
    tree = ast.parse(src)
    found = {}
    scopes = [tree]
    if nested_in:
        for node in ast.walk(tree):
            if isinstance(node, ast.FunctionDef) and node.name == nested_in:
                scopes = [node]
    for scope in scopes:
        for node in ast.walk(scope):
            if isinstance(node, ast.FunctionDef) and node.name in names:
                node.decorator_list = []
                found[node.name] = node
            if isinstance(node, ast.Assign) and len(node.targets) == 1:
                tgt = node.targets[0]
                tnames = [tgt.id] if isinstance(tgt, ast.Name) else \
                    [e.id for e in getattr(tgt, "elts", []) if isinstance(e, ast.Name)]
                for tn in tnames:
                    if tn in names:
                        found[tn] = node
    missing = set(names) - set(found)
    if missing:
        raise KeyError(f"{path}: not found {missing}")
    return [found[n] for n in names]


class Reference:
    """Namespace holding the extracted reference functions."""

    def __init__(self, root):
        self.root = root
        ns = dict(torch=torch, F=F, Tensor=torch.Tensor, functools=functools,
                  Optional=__import__("typing").Optional, Tuple=__import__("typing").Tuple,
                  dtypes=_dtypes_ns(), ActivationType=ActivationType, QuantType=QuantType,
                  BLOCK_SIZE_M=32)
        self.ns = ns
        # fp4 codecs first: quant and the stage functions use them
        fp4 = self._load(ns, "aiter/utility/fp4_utils.py",
                         ["_n_ones", "EBITS_F32", "F32_EXP_BIAS", "_f32_to_floatx_unpacked", "down_size", "pack_uint4",
                          "f32_to_mxfp4", "mxfp4_to_f32", "f32_to_e8m0", "e8m0_to_f32", "e8m0_shuffle"])
        fp4_mod = types.ModuleType("fp4_utils")
        for k in fp4 + ["MBITS_F32"]:
            setattr(fp4_mod, k, ns[k])
        ns["fp4_utils"] = fp4_mod
        self._load(ns, "aiter/ops/quant.py", ["get_dtype_max", "pertoken_quant", "per_1x32_f4_quant"])
        aiter_ns = types.SimpleNamespace(ActivationType=ActivationType, QuantType=QuantType,
                                         get_torch_act=_get_torch_act,
                                         pertoken_quant=ns["pertoken_quant"])
        ns["aiter"] = aiter_ns
        self._load(ns, "aiter/fused_moe.py",
                   ["quant_remap", "get_inter_dim", "swiglu", "torch_moe_act", "torch_moe",
                    "torch_moe_stage1", "torch_moe_stage2"])
        self._load(ns, "aiter/ops/topk.py", ["biased_grouped_topk_torch", "grouped_topk_torch"])
        self._load(ns, "op_tests/test_moe_sorting.py", ["moe_sorting_native"])
        self._load(ns, "aiter/ops/shuffle.py", ["shuffle_weight"])
        # the torch reference of the sorted MXFP4 scale layout, kept under its own name
        run_torch = dict(torch=torch)
        self._load(run_torch, "op_tests/test_moe_sorting_mxfp4.py", ["run_torch"])
        ns["moe_mxfp4_sort_torch"] = run_torch["run_torch"]
        self._load(ns, "op_tests/test_moeTopkSoftmax.py", ["test_nofuse"])
        # torch references of topk_sigmoid and silu_and_mul, kept under their own names
        ts = dict(torch=torch)
        self._load(ts, "op_tests/test_moe_topk_sigmoid.py", ["run_torch"])
        ns["topk_sigmoid_torch"] = ts["run_torch"]
        self._load(ns, "op_tests/test_activation.py", ["torch_silu_and_mul"])
        self._load(ns, "op_tests/test_moe_2stage.py", ["weight_per_128x128_quant"],
                   nested_in="test_fmoe")
        self._load(ns, "op_tests/test_moe_blockscale.py", ["torch_moe_blockscale"])
        ns["rearrange"] = __import__("einops").rearrange
        for k, v in ns.items():
            setattr(self, k, v)

    def _load(self, ns, rel, names, nested_in=None):
        nodes = _extract(f"{self.root}/{rel}", names, nested_in)
        mod = ast.Module(body=nodes, type_ignores=[])
        ast.fix_missing_locations(mod)
        # `from aiter.utility import fp4_utils` inside the stage functions
        aiter_pkg = types.ModuleType("aiter")
        util_pkg = types.ModuleType("aiter.utility")
        saved = {k: sys.modules.get(k) for k in ("aiter", "aiter.utility")}
        if "fp4_utils" in ns:
            util_pkg.fp4_utils = ns["fp4_utils"]
            aiter_pkg.utility = util_pkg
            sys.modules["aiter"], sys.modules["aiter.utility"] = aiter_pkg, util_pkg
        try:
            exec(compile(mod, f"{self.root}/{rel}", "exec"), ns)
        finally:
            for k, v in saved.items():
                if v is None:
                    sys.modules.pop(k, None)
                else:
                    sys.modules[k] = v
        return names

    def call_with_fp4_module(self, fn, *a, **k):
        """Run a function that may `from aiter.utility import fp4_utils` at call time."""
        aiter_pkg = types.ModuleType("aiter")
        util_pkg = types.ModuleType("aiter.utility")
        util_pkg.fp4_utils = self.ns["fp4_utils"]
        aiter_pkg.utility = util_pkg
        saved = {k: sys.modules.get(k) for k in ("aiter", "aiter.utility")}
        sys.modules["aiter"], sys.modules["aiter.utility"] = aiter_pkg, util_pkg
        try:
            return fn(*a, **k)
        finally:
            for kk, v in saved.items():
                if v is None:
                    sys.modules.pop(kk, None)
                else:
                    sys.modules[kk] = v
