"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configs.

The reference measures on no public dataset; these generators stand in for its inputs. CPU
generation (torch's CPU generator) is deterministic across machines for a given torch version, so
tests regenerate inputs from the seed and the committed fixtures hold only outputs plus an input
checksum that proves the regeneration matches.
"""
import hashlib

import torch


def checksum(*ts) -> str:
    h = hashlib.sha256()
    for t in ts:
        if t is None:
            h.update(b"none")
            continue
        t = t.detach().cpu().contiguous()
        h.update(str(tuple(t.shape)).encode() + str(t.dtype).encode())
        h.update(t.view(torch.uint8).numpy().tobytes() if t.numel() else b"")
    return h.hexdigest()[:16]


def config1(seed=0):
    """Config 1: X [256,1024] bf16, rows N(0,1) * 2^r with r ~ U{-12..18}; W [1024,1024] N(0, 0.02^2);
    bias [1024] N(0, 0.01^2)."""
    g = torch.Generator().manual_seed(seed)
    r = torch.randint(-12, 19, (256,), generator=g)
    x = (torch.randn(256, 1024, generator=g) * torch.pow(2.0, r.float())[:, None]).bfloat16()
    w = (torch.randn(1024, 1024, generator=g) * 0.02).bfloat16()
    b = (torch.randn(1024, generator=g) * 0.01).bfloat16()
    return x, w, b


def gemm_x(M, K, seed=0, device="cpu", outlier_frac=0.02):
    """Config 2 activations: N(0,1) entries, row magnitudes 2^u with u ~ U(-16, 20), and 2% of the
    input channels multiplied by 2^12."""
    g = torch.Generator(device=device).manual_seed(seed)
    u = torch.rand(M, 1, generator=g, device=device) * 36.0 - 16.0
    x = torch.randn(M, K, generator=g, device=device) * torch.exp2(u)
    n_out = max(1, int(round(K * outlier_frac)))
    ch = torch.randperm(K, generator=g, device=device)[:n_out]
    x[:, ch] *= 2.0 ** 12
    return x.bfloat16()


def gemm_w(N, K, seed=1, device="cpu"):
    """Config 2 weights: N(0, 1/K)."""
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(N, K, generator=g, device=device) * K ** -0.5).bfloat16()


def attention_qkv(B, H, S, D, seed=0, device="cpu", Hkv=None, qk_exp=8, v_exp_max=14):
    """Config 3: Q, K entries N(0,1) * 2^8 (raw logits overflow fp16); V entries N(0,1) * 2^h with
    h ~ U{0..14} per head."""
    Hkv = Hkv or H
    g = torch.Generator(device=device).manual_seed(seed)
    q = (torch.randn(B, H, S, D, generator=g, device=device) * 2.0 ** qk_exp).bfloat16()
    k = (torch.randn(B, Hkv, S, D, generator=g, device=device) * 2.0 ** qk_exp).bfloat16()
    h = torch.randint(0, v_exp_max + 1, (B, Hkv, 1, 1), generator=g, device=device).float()
    v = (torch.randn(B, Hkv, S, D, generator=g, device=device) * torch.exp2(h)).bfloat16()
    return q, k, v
