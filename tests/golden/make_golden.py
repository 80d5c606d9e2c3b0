"""Generate golden vectors by running the REFERENCE's own code (tech-cosmos/turing-bf16) on CPU.

Run where the reference checkout is available (TBF16_REFERENCE, default: a `reference` directory
beside this repository). Its CUDA kernels need a GPU, but its Triton kernels run on CPU under
TRITON_INTERPRET=1 and its torch fallbacks run on CPU with tbf16.ops._USE_CUDA = False, so these
reference code paths produce the fixtures:
  - ops.quantize_rows / ops.prepare_weight        (Triton _quantize_rows_kernel, ops.py:48-89)
  - ops.scaled_linear for 2 <= M < 256 and config 1 (quantize L1 t=15 -> fp16 GEMM -> Triton
    epilogue, ops.py:153-178; torch's CPU fp16 matmul stands in for cuBLAS)
  - attention.head_exp / head_scale / prepare_qkv / sdpa   (torch fallbacks, attention.py:24-65)
  - autograd.quantize_cols                          (torch fallback, autograd.py:26-36)
  - ops._target_exp
Inputs are regenerated from seeds in the tests; each fixture stores the outputs and an input
checksum. Writes tests/golden/golden.npz.

    python tests/golden/make_golden.py
"""
import os
import pathlib
import sys

os.environ["TRITON_INTERPRET"] = "1"
HERE = pathlib.Path(__file__).resolve().parent
REF = os.environ.get("TBF16_REFERENCE", str(HERE.parents[2] / "reference"))
sys.path.insert(0, REF)
sys.path.insert(0, str(HERE))

import numpy as np  # noqa: E402
import torch  # noqa: E402

import inputs  # noqa: E402
import tbf16.attention as ref_att  # noqa: E402
import tbf16.autograd as ref_ag  # noqa: E402
import tbf16.ops as ref_ops  # noqa: E402

ref_ops._USE_CUDA = False


def u16(t):
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


def rows_case(seed, R, K):
    """bf16 rows spanning many binades, with edge rows: zero, single huge element, tiny values."""
    g = torch.Generator().manual_seed(seed)
    e = torch.randint(-30, 31, (R, 1), generator=g).float()
    x = torch.randn(R, K, generator=g) * torch.exp2(e)
    x[0] = 0.0
    x[1, :] = 1e-3
    x[1, 3] = 3e4
    x[2] = torch.exp2(torch.randint(-20, 20, (K,), generator=g).float())  # exact powers of two
    return x.bfloat16()


def main():
    out = {}
    # _target_exp (ops.py:29-32)
    Ks = [1, 2, 7, 8, 100, 1024, 4096, 32768, 32769, 65536, 65537, 131072, 1 << 20]
    out["target_exp_K"] = np.array(Ks, dtype=np.int64)
    out["target_exp_t"] = np.array([ref_ops._target_exp(k) for k in Ks], dtype=np.int64)

    # quantize_rows through the reference's Triton kernel (one-pass K <= 16384 and two-pass K > 16384)
    for i, (R, K) in enumerate([(16, 64), (8, 1032), (3, 20000)]):
        x = rows_case(100 + i, R, K)
        out[f"qr{i}_meta"] = np.array([100 + i, R, K])
        out[f"qr{i}_xsum"] = np.array(inputs.checksum(x))
        for t in (0, -1, 15):
            for l1 in (False, True):
                y, s = ref_ops.quantize_rows(x, t, l1)
                out[f"qr{i}_t{t}_l{int(l1)}_y"] = u16(y)
                out[f"qr{i}_t{t}_l{int(l1)}_s"] = s.numpy()

    # prepare_weight (ops.py:140-142)
    w = inputs.gemm_w(96, 1024, seed=7)
    w16, ws = ref_ops.prepare_weight(w)
    out["pw_xsum"] = np.array(inputs.checksum(w))
    out["pw_w16"], out["pw_ws"] = u16(w16), ws.numpy()

    # scaled_linear small-M default path (ops.py:163-164): M = 4, 33, 130
    for i, M in enumerate([4, 33, 130]):
        x = inputs.gemm_x(M, 512, seed=20 + i)
        w = inputs.gemm_w(256, 512, seed=30 + i)
        b = (torch.randn(256, generator=torch.Generator().manual_seed(40 + i)) * 0.1).bfloat16()
        w16, ws = ref_ops.prepare_weight(w)
        y = ref_ops.scaled_linear(x, w16, ws, b)
        out[f"sl{i}_meta"] = np.array([M, 512, 256, 20 + i, 30 + i, 40 + i])
        out[f"sl{i}_xsum"] = np.array(inputs.checksum(x, w, b))
        out[f"sl{i}_y"] = u16(y)

    # config 1 through the reference's CPU-runnable path (M = 256 would use the fused CUDA kernel on a
    # GPU; without CUDA the reference takes quantize + fp16 GEMM + epilogue).
    x, w, b = inputs.config1()
    w16, ws = ref_ops.prepare_weight(w)
    y = ref_ops.scaled_linear(x, w16, ws, b)
    out["c1_xsum"] = np.array(inputs.checksum(x, w, b))
    out["c1_w16sum"], out["c1_ws"], out["c1_y"] = np.array(inputs.checksum(w16)), ws.numpy(), u16(y)

    # quantize_cols torch fallback (autograd.py:26-36), with and without row_mul
    x = rows_case(200, 48, 64)
    rm = torch.exp2(torch.randint(-8, 9, (48,), generator=torch.Generator().manual_seed(201)).float())
    out["qc_xsum"] = np.array(inputs.checksum(x, rm))
    for t in (0, -3):
        y, s = ref_ag.quantize_cols(x, t)
        out[f"qc_t{t}_y"], out[f"qc_t{t}_s"] = u16(y), s.numpy()
        y, s = ref_ag.quantize_cols(x, t, rm)
        out[f"qcm_t{t}_y"], out[f"qcm_t{t}_s"] = u16(y), s.numpy()

    # attention helpers and inference sdpa (attention.py:24-65) on CPU
    cases = [(1, 2, 64, 64, 2, False, 8), (2, 4, 48, 32, 2, True, 8), (1, 4, 80, 128, 4, False, 12)]
    for i, (B, H, S, D, Hkv, causal, qk) in enumerate(cases):
        q, k, v = inputs.attention_qkv(B, H, S, D, seed=300 + i, Hkv=Hkv, qk_exp=qk)
        out[f"at{i}_meta"] = np.array([B, H, S, D, Hkv, int(causal), qk, 300 + i])
        out[f"at{i}_xsum"] = np.array(inputs.checksum(q, k, v))
        out[f"at{i}_eq"] = ref_att.head_exp(q).numpy()
        out[f"at{i}_amax_q"] = q.abs().amax(dim=(-2, -1)).float().numpy()
        for v_exp in (0, 13):
            q16, k16, v16, a, ev = ref_att.prepare_qkv(q, k, v, v_exp=v_exp)
            out[f"at{i}_v{v_exp}_q16"], out[f"at{i}_v{v_exp}_k16"], out[f"at{i}_v{v_exp}_v16"] = u16(q16), u16(k16), u16(v16)
            out[f"at{i}_v{v_exp}_a"], out[f"at{i}_v{v_exp}_ev"] = np.array(int(a)), ev.numpy()
        o = ref_att.sdpa(q, k, v, is_causal=causal, enable_gqa=Hkv != H)
        out[f"at{i}_out"] = u16(o)
        # head_scale on a bf16 tensor with negative and positive exponents
        e = torch.arange(B * H, dtype=torch.int32).view(B, H) - 3
        out[f"at{i}_hs"] = u16(ref_att.head_scale(q, e, torch.float16))

    np.savez_compressed(HERE / "golden.npz", **out)
    print(f"wrote {len(out)} arrays to {HERE / 'golden.npz'}")


if __name__ == "__main__":
    main()
