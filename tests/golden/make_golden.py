"""Generates the golden vectors that pin the CPU oracle's attention and cache-write semantics.

The reference reaches decode attention and the cache write through vLLM 0.5.1 (un-vendored; its
FlashAttention backend calls ``reshape_and_cache_flash`` then ``flash_attn_with_kvcache`` with a
block table). This script runs the same kernel family from the installed vLLM 0.22 on a GPU:
``vllm._custom_ops.reshape_and_cache_flash`` and ``vllm.vllm_flash_attn.flash_attn_varlen_func``
(FA2, ``block_table`` + ``seqused_k``, causal, one query token per sequence) on the cfg1 shape
(Qwen2.5-7B attention: 28 query heads, 4 KV heads, head_dim 128, fp16, block size 16) and on a
bf16 GQA-8 case, over per-layer views of Aegaeon's interleaved (N, L, 2, 16, Hkv, D) cache, and
saves the inputs, vLLM's attention output and the SHA-256 of the cache after vLLM's write to
``tests/golden/*.npz``. The prompt cases run ``flash_attn_varlen_func(..., causal=True)`` on the
q/k/v of whole prompts (the backend's prompt call) and save inputs and output.

Run on a CUDA machine with vLLM installed:  python tests/golden/make_golden.py
Only this generator touches vLLM; the tests read the saved arrays.
"""
from __future__ import annotations

import hashlib
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _case(name, B, Hq, Hkv, ctx_lo, ctx_hi, n_blocks, L, dtype, seed, out_dir):
    from vllm import _custom_ops as vops
    from vllm.vllm_flash_attn import flash_attn_varlen_func

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(ctx_lo, ctx_hi + 1, (B,), generator=g)
    nb = (ctx + 15) // 16
    assert int(nb.sum()) <= n_blocks
    perm = torch.randperm(n_blocks, generator=g)
    W = int(nb.max())
    tables = torch.zeros((B, W), dtype=torch.int32)
    off = 0
    for b in range(B):
        tables[b, : nb[b]] = perm[off: off + nb[b]].to(torch.int32)
        off += int(nb[b])
    D = 128
    cache = torch.randn((n_blocks, L, 2, 16, Hkv, D), generator=g).to(dtype)
    q = torch.randn((B, Hq, D), generator=g).to(dtype)
    k_new = torch.randn((B, Hkv, D), generator=g).to(dtype)
    v_new = torch.randn((B, Hkv, D), generator=g).to(dtype)
    layer = L - 1
    # decode slots: position ctx-1 of each sequence; one padding slot (-1) to check it is skipped
    pos = ctx - 1
    slots = (tables[torch.arange(B), pos // 16].to(torch.int64) * 16 + pos % 16)
    slots_in = slots.clone()
    slots_in[0] = -1

    cache_d = cache.to(dev)
    run = cache_d.permute(1, 2, 0, 3, 4, 5)  # (L, 2, N, 16, Hkv, D) as the reference's worker
    kc, vc = run[layer][0], run[layer][1]
    one = torch.ones((), dtype=torch.float32, device=dev)
    vops.reshape_and_cache_flash(k_new.to(dev), v_new.to(dev), kc, vc, slots_in.to(dev), "auto", one, one)
    torch.cuda.synchronize()
    cache_after = cache_d.cpu()

    scale = 1.0 / math.sqrt(D)
    out = flash_attn_varlen_func(
        q=q.to(dev), k=kc, v=vc, max_seqlen_q=1,
        cu_seqlens_q=torch.arange(B + 1, dtype=torch.int32, device=dev), max_seqlen_k=int(ctx.max()),
        seqused_k=ctx.to(torch.int32).to(dev), softmax_scale=scale, causal=True,
        block_table=tables.to(dev), fa_version=2)
    torch.cuda.synchronize()
    u16 = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
    path = os.path.join(out_dir, f"{name}.npz")
    after = u16(cache_after)
    np.savez_compressed(
        path, q=u16(q), cache_before=u16(cache), cache_after_sha256=np.array(hashlib.sha256(after.tobytes()).hexdigest()),
        k_new=u16(k_new), v_new=u16(v_new),
        slot_mapping=slots_in.numpy(), tables=tables.numpy(), seq_lens=ctx.to(torch.int32).numpy(),
        out_vllm=u16(out.cpu()), layer=np.int32(layer), num_kv_heads=np.int32(Hkv),
        dtype=np.array("bf16" if dtype == torch.bfloat16 else "fp16"), scale=np.float64(scale),
        generator=np.array("vllm %s reshape_and_cache_flash + vllm_flash_attn.flash_attn_varlen_func(fa_version=2)"
                           % __import__("vllm").__version__))
    print("wrote", path)


def _prefill_case(name, lens, Hq, Hkv, dtype, seed, out_dir):
    """Prompt attention: vLLM's varlen FlashAttention on q/k/v of whole prompts, causal (the call
    the reference's backend makes for prompts, Aegaeon prefilling without chunking)."""
    from vllm.vllm_flash_attn import flash_attn_varlen_func

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(seed)
    T, D = int(sum(lens)), 128
    q = torch.randn((T, Hq, D), generator=g).to(dtype)
    k = torch.randn((T, Hkv, D), generator=g).to(dtype)
    v = torch.randn((T, Hkv, D), generator=g).to(dtype)
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    scale = 1.0 / math.sqrt(D)
    out = flash_attn_varlen_func(q=q.to(dev), k=k.to(dev), v=v.to(dev), cu_seqlens_q=cu.to(dev),
                                 cu_seqlens_k=cu.to(dev), max_seqlen_q=max(lens), max_seqlen_k=max(lens),
                                 softmax_scale=scale, causal=True, fa_version=2)
    torch.cuda.synchronize()
    u16 = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
    path = os.path.join(out_dir, f"{name}.npz")
    np.savez_compressed(
        path, q=u16(q), k=u16(k), v=u16(v), cu_seqlens=cu.numpy(), out_vllm=u16(out.cpu()),
        dtype=np.array("bf16" if dtype == torch.bfloat16 else "fp16"), scale=np.float64(scale),
        generator=np.array("vllm %s vllm_flash_attn.flash_attn_varlen_func(causal=True, fa_version=2)"
                           % __import__("vllm").__version__))
    print("wrote", path)


def main(out_dir: str = HERE) -> None:
    _case("vllm_cfg1_fp16", 4, 28, 4, 17, 300, 64, 1, torch.float16, 0, out_dir)
    _case("vllm_gqa8_bf16", 6, 32, 4, 1, 400, 160, 1, torch.bfloat16, 1, out_dir)
    _prefill_case("vllm_prefill_fp16", [1, 17, 65, 130], 4, 1, torch.float16, 2, out_dir)
    _prefill_case("vllm_prefill_bf16", [1, 17, 65, 130], 4, 1, torch.bfloat16, 3, out_dir)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
