"""Element types of the path (aiter/utility/dtypes.py): fp8 is the OCP
float8_e4m3fn on NVIDIA hardware (max 448), fp4x2 packs two e2m1 values per byte
with element 2i in the low nibble, fp8_e8m0 is the power-of-two scale type."""
import torch

fp8 = torch.float8_e4m3fn
fp8_e8m0 = torch.float8_e8m0fnu
fp4x2 = torch.float4_e2m1fn_x2
fp16 = torch.float16
bf16 = torch.bfloat16
fp32 = torch.float32
i32 = torch.int32
i8 = torch.int8
u8 = torch.uint8
u32 = torch.uint32

FP8_MAX = 448.0

d_dtypes = {"fp8": fp8, "fp8_e8m0": fp8_e8m0, "fp4x2": fp4x2, "fp16": fp16, "bf16": bf16,
            "fp32": fp32, "i32": i32, "i8": i8, "u8": u8, "u32": u32}


def str2Dtype(s):
    return d_dtypes[s]
