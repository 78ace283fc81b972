"""Generates golden vectors that pin the step-input oracle (``oracle.np_step_inputs``) to the
reference's own code.

The reference builds each step's slot mapping, positions, start offsets and attention table rows
in ``Worker._prepare_model_inputs`` (aegaeon/aegaeon/worker.py:554-713), padding the table rows
with ``make_tensor_with_pad`` (aegaeon/aegaeon/utils.py:241-257). Their modules cannot be
imported whole here (worker.py needs ray, viztracer and vLLM 0.5.1's internals), so this script
compiles those two functions from the reference's source files, as they are, into a namespace
with numpy and torch, and calls the method with a stand-in ``self`` that supplies what it reads:
the block size (16), a CPU device, a model config without logit soft-capping, and an attention
backend whose ``make_metadata`` returns its arguments. Nothing of the reference is copied into
this repository; the saved arrays are its outputs on seeded batches (prompts first, then decode
requests, as the method requires).

Run in a checkout with the reference beside it:
    python tests/golden/make_step_inputs_golden.py [path/to/reference/aegaeon]
Only this generator reads the reference; the tests read ``step_inputs_reference.npz``.
"""
from __future__ import annotations

import ast
import os
import sys
import textwrap
import types
from typing import List, Optional, Tuple, Union

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT_REF = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(HERE))), "reference", "aegaeon")


def _function_source(path: str, name: str, cls: str | None = None) -> str:
    tree = ast.parse(open(path).read())
    scope = tree.body
    if cls is not None:
        scope = next(n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == cls).body
    node = next(n for n in scope if isinstance(n, ast.FunctionDef) and n.name == name)
    return textwrap.dedent(ast.get_source_segment(open(path).read(), node))


def load_reference(ref_dir: str):
    pkg = os.path.join(ref_dir, "aegaeon")
    ns = {"np": np, "torch": torch, "List": List, "Optional": Optional, "Tuple": Tuple, "Union": Union,
          "RequestMeta": Tuple[int, List[int], int, int]}
    exec(compile(_function_source(os.path.join(pkg, "utils.py"), "make_tensor_with_pad"), "utils.py", "exec"), ns)
    exec(compile(_function_source(os.path.join(pkg, "worker.py"), "_prepare_model_inputs", "Worker"), "worker.py",
                 "exec"), ns)
    return ns["_prepare_model_inputs"]


def _stand_in_worker():
    return types.SimpleNamespace(
        block_size=16, device="cpu",
        model_config=types.SimpleNamespace(hf_config=types.SimpleNamespace()),
        attn_backend=types.SimpleNamespace(make_metadata=lambda **kw: kw))


def _batch(rng, n_prompts, n_decode, max_len):
    """Prompts (context 0) first, then decode requests (one new token), each with its own blocks."""
    perm = rng.permutation(1 << 16)
    reqs, tables, off = [], [], 0
    for i in range(n_prompts + n_decode):
        n = int(rng.integers(1, max_len + 1))
        c = 0 if i < n_prompts else n - 1
        nb = (n + 15) // 16
        tables.append([int(b) for b in perm[off:off + nb]])
        off += nb
        reqs.append((i, list(range(n - c)), n, c))
    return reqs, tables


def main():
    ref_dir = sys.argv[1] if len(sys.argv) > 1 else DEFAULT_REF
    prepare = load_reference(ref_dir)
    rng = np.random.default_rng(2024)
    out = {}
    cases = [(0, 5, 300), (3, 0, 700), (4, 60, 2000), (1, 1, 16), (16, 240, 4096)]
    for k, (n_prompts, n_decode, max_len) in enumerate(cases):
        reqs, tables = _batch(rng, n_prompts, n_decode, max_len)
        tokens, positions, md = prepare(_stand_in_worker(), reqs, tables)
        out[f"c{k}_seq_lens"] = np.asarray([r[2] for r in reqs], np.int32)
        out[f"c{k}_context_lens"] = np.asarray([r[3] for r in reqs], np.int32)
        out[f"c{k}_table_offsets"] = np.concatenate([[0], np.cumsum([len(t) for t in tables])]).astype(np.int64)
        out[f"c{k}_tables_flat"] = np.asarray([b for t in tables for b in t], np.int32)
        out[f"c{k}_positions"] = positions.numpy().astype(np.int64)
        out[f"c{k}_slot_mapping"] = md["slot_mapping"].numpy().astype(np.int64)
        out[f"c{k}_query_start_loc"] = md["query_start_loc"].numpy().astype(np.int32)
        out[f"c{k}_seq_start_loc"] = md["seq_start_loc"].numpy().astype(np.int32)
        out[f"c{k}_block_tables"] = md["block_tables"].numpy().astype(np.int32)
        out[f"c{k}_max_query_len"] = np.asarray(md["max_query_len"], np.int64)
    out["cases"] = np.asarray(len(cases), np.int64)
    path = os.path.join(HERE, "step_inputs_reference.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
