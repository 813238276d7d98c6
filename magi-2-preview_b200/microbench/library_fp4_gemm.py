"""One library NVFP4 GEMM shape (cuBLASLt through torch._scaled_mm), three launches: the
case an ncu capture of the library's kernel runs.

    python magi-2-preview_b200/microbench/library_fp4_gemm.py [M N K]   # default 32768 2048 3072
"""
import sys
import torch
M, N, K = (int(v) for v in (sys.argv[1:4] if len(sys.argv) > 3 else (32768, 2048, 3072)))
dev = torch.device("cuda", 0)
g = torch.Generator(device=dev).manual_seed(0)
a = torch.randint(0, 256, (M, K // 2), dtype=torch.uint8, device=dev, generator=g).view(torch.float4_e2m1fn_x2)
b = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev, generator=g).view(torch.float4_e2m1fn_x2)
rup = lambda v, m: (v + m - 1) // m * m
sa = torch.full((rup(M, 128) * rup(K // 16, 4),), 1.0, device=dev).to(torch.float8_e4m3fn)
sb = torch.full((rup(N, 128) * rup(K // 16, 4),), 1.0, device=dev).to(torch.float8_e4m3fn)
for _ in range(3):
    out = torch._scaled_mm(a, b.t(), sa, sb, out_dtype=torch.bfloat16)
torch.cuda.synchronize()
print("ok", out.shape)
