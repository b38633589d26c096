"""Regenerate the golden vectors in this folder from the REFERENCE's own code.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py --reference /path/to/reference

It imports the reference's ground-truth functions from ``base/``
(``baseline_gqa.fp64_reference``, ``baseline_gqa_causal.fp64_reference_causal``,
``baseline_gqa_split.fp64_reference``, ``baseline_mha.fp64_attention`` and the
``sdpa_gqa*`` torch-SDPA calls), sets the module globals those functions read
(B, Hq, G, S / Sq / Skv, D; base/baseline_gqa.py:29-30), runs them on CPU
tensors and writes one ``.npz`` per case.  bf16 inputs are stored as their raw
16-bit patterns (uint16) so the GPU tests feed the kernel exactly the bits the
reference saw; fp32 inputs are stored as float32.

The GPU box does not have the reference: tests only read the ``.npz`` files.
"""
import argparse
import importlib.util
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def load(ref_root: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, ref_root / "base" / f"{name}.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def gen(shape, dist, gen_):
    if dist == "randn":
        return torch.randn(*shape, generator=gen_, dtype=torch.float32)
    return torch.rand(*shape, generator=gen_, dtype=torch.float32)


def case_gqa(mod_gqa, mod_causal, name, B, Hq, Hkv, S, D, causal, dist, bf16=True):
    g = torch.Generator().manual_seed(42)
    q, k, v = gen((B, Hq, S, D), dist, g), gen((B, Hkv, S, D), dist, g), gen((B, Hkv, S, D), dist, g)
    if bf16:
        q, k, v = q.bfloat16().float(), k.bfloat16().float(), v.bfloat16().float()
    scale = 1.0 / math.sqrt(D)
    mod = mod_causal if causal else mod_gqa
    mod.B, mod.Hq, mod.Hkv, mod.S, mod.D, mod.G = B, Hq, Hkv, S, D, Hq // Hkv
    if causal:
        o64, lse64 = mod.fp64_reference_causal(q, k, v, scale)
        osd = mod.sdpa_gqa_causal(q, k, v, scale)
    else:
        o64, lse64 = mod.fp64_reference(q, k, v, scale)
        osd = mod.sdpa_gqa(q, k, v, scale)
    out = dict(scale=np.float32(scale), causal=np.int32(causal), o_fp64=o64.numpy(),
               lse_fp64=lse64.numpy())
    if not bf16:  # the fp32 plumbing case also pins the SDPA (CPU execution) path
        out["o_sdpa"] = osd.float().numpy()
    if bf16:
        out.update(q_bf16=bf16_bits(q), k_bf16=bf16_bits(k), v_bf16=bf16_bits(v))
    else:
        out.update(q_f32=q.numpy(), k_f32=k.numpy(), v_f32=v.numpy())
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(name, {k_: v_.shape for k_, v_ in out.items()})


def case_split(mod, name, B, Hq, Hkv, Sq, Skv, D, dist):
    g = torch.Generator().manual_seed(42)
    q = gen((B, Hq, Sq, D), dist, g).bfloat16().float()
    k = gen((B, Hkv, Skv, D), dist, g).bfloat16().float()
    v = gen((B, Hkv, Skv, D), dist, g).bfloat16().float()
    scale = 1.0 / math.sqrt(D)
    mod.B, mod.Hq, mod.Hkv, mod.Sq, mod.Skv, mod.D, mod.G = B, Hq, Hkv, Sq, Skv, D, Hq // Hkv
    o64, lse64 = mod.fp64_reference(q, k, v, scale)
    osd = mod.sdpa_gqa(q, k, v, scale)
    np.savez_compressed(HERE / f"{name}.npz", scale=np.float32(scale), causal=np.int32(0),
                        q_bf16=bf16_bits(q), k_bf16=bf16_bits(k), v_bf16=bf16_bits(v),
                        o_fp64=o64.numpy(), lse_fp64=lse64.numpy())
    print(name)


def case_mha(mod, name, B, H, S, D):
    g = torch.Generator().manual_seed(42)
    # baseline_mha.py:71-73 draws U[0,1) - 0.5 in fp32
    q, k, v = [(torch.rand(B, H, S, D, generator=g) - 0.5) for _ in range(3)]
    scale = 1.0 / math.sqrt(D)
    o64 = mod.fp64_attention(q, k, v, scale)
    np.savez_compressed(HERE / f"{name}.npz", scale=np.float32(scale), q_f32=q.numpy(),
                        k_f32=k.numpy(), v_f32=v.numpy(), o_fp64=o64.numpy())
    print(name)


def case_decode(mod, name, B, Hq, Hkv, D, lens):
    """Single-token decode: the split-length reference with Sq=1, Skv=L_b, per sequence."""
    g = torch.Generator().manual_seed(42)
    total = int(sum(lens))
    q = torch.randn(B, Hq, D, generator=g).bfloat16().float()
    k = torch.randn(total, Hkv, D, generator=g).bfloat16().float()
    v = torch.randn(total, Hkv, D, generator=g).bfloat16().float()
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    scale = 1.0 / math.sqrt(D)
    o = np.zeros((B, Hq, D), np.float32)
    lse = np.zeros((B, Hq), np.float32)
    for b in range(B):
        L = int(lens[b])
        s0 = int(offs[b])
        mod.B, mod.Hq, mod.Hkv, mod.Sq, mod.Skv, mod.D, mod.G = 1, Hq, Hkv, 1, L, D, Hq // Hkv
        qb = q[b][None, :, None, :]                                  # [1, Hq, 1, D]
        kb = k[s0:s0 + L].permute(1, 0, 2)[None]                     # [1, Hkv, L, D]
        vb = v[s0:s0 + L].permute(1, 0, 2)[None]
        ob, lb = mod.fp64_reference(qb, kb, vb, scale)
        o[b] = ob[0, :, 0].numpy()
        lse[b] = lb[0, :, 0].numpy()
    np.savez_compressed(HERE / f"{name}.npz", scale=np.float32(scale), q_bf16=bf16_bits(q),
                        k_bf16=bf16_bits(k), v_bf16=bf16_bits(v), kv_lens=np.asarray(lens, np.int32),
                        kv_offsets=offs, o_fp64=o, lse_fp64=lse)
    print(name)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=str(Path(__file__).resolve().parents[3] / "reference"),
                    help="the reference checkout (default: next to this repository)")
    args = ap.parse_args()
    ref = Path(args.reference)
    sys.path.insert(0, str(ref / "base"))
    m_gqa = load(ref, "baseline_gqa")
    m_causal = load(ref, "baseline_gqa_causal")
    m_split = load(ref, "baseline_gqa_split")
    m_mha = load(ref, "baseline_mha")
    # C1: the CPU plumbing config exactly (fp32, N(0,1), non-causal).
    case_gqa(m_gqa, m_causal, "c1_gqa_fp32", 1, 8, 2, 512, 64, False, "randn", bf16=False)
    # bf16 cases for the GPU kernel (N(0,1) per the configs; U[0,1) per the reference scripts).
    case_gqa(m_gqa, m_causal, "gqa_nc_d128", 1, 4, 2, 256, 128, False, "randn")
    case_gqa(m_gqa, m_causal, "gqa_causal_d128", 1, 4, 1, 320, 128, True, "randn")
    case_gqa(m_gqa, m_causal, "gqa_causal_d64_g3_rand", 1, 6, 2, 256, 64, True, "rand")
    case_gqa(m_gqa, m_causal, "gqa_causal_d64_ragged", 2, 2, 2, 200, 64, True, "randn")
    case_split(m_split, "gqa_split_d64", 1, 4, 2, 200, 328, 64, "randn")
    case_mha(m_mha, "mha_fp32_d64", 2, 2, 256, 64)
    case_decode(m_split, "decode_d128", 4, 16, 2, 128, [1, 37, 300, 1029])


if __name__ == "__main__":
    main()
