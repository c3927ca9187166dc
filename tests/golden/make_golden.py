"""Generate the golden fixtures in this folder from the reference's own Python modules.

Run where a checkout of runwangdl/softhier-mlir is available, with SOFTHIER_REF set to its path:

    SOFTHIER_REF=<checkout> python tests/golden/make_golden.py

It imports the reference's host-side code, never this repository's oracle, and writes:
  lcg.npz            draws of softhier_mlir.testing.lcg._lcg_stream, fill_fp16 / const / col-parity
                     fills and sample_positions for a spread of seeds, sizes and ranges
  siglip_small.npz   every tensor of siglip_ref.layer_reference at two small shapes
  siglip_s256.npz    siglip_ref.layer_reference(256, 768, 3072, 12) sampled at the frontend's dump
                     positions (64 samples per tensor) plus per-tensor float64 sums
  attention.npz      tests/gvsoc/run.py attention_reference at two shapes (inputs + output)
  preload_small.elf  a small HBM preload image written by sim/preload.make_preload_elf (3 arrays + sentinel),
  preload_small.npz  its segments as sim/preload.read_preload_elf returns them
  llm.npz            the decoder ops' numpy twins of frontend/smolvla_expert.py (rmsnorm, rope, silu-mul,
                     GQA attention with a padding-token mask) and frontend/smolvla.py (rope table, pixel shuffle)
  mlir/*.mlir        frontend/siglip.emit output for the configurations the emitter tests lower
The parity tests read only these files at run time.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _ref_root() -> Path:
    """The reference checkout (runwangdl/softhier-mlir) named by SOFTHIER_REF."""
    if not os.environ.get("SOFTHIER_REF"):
        raise SystemExit("set SOFTHIER_REF to a checkout of the reference (runwangdl/softhier-mlir)")
    return Path(os.environ["SOFTHIER_REF"])


def _q_block_rule(S: int, dh: int, H: int, cluster: int) -> int:
    """The q-block rule the frontend asks softhier_mlir.dse.tiling for (sh_attention.inc.c:55-65), restated
    because that module imports xdsl: the largest sq in {S, 256, 128, 64} dividing S whose TCDM layout
    (sh_attention.inc.c:43-49, base 0x1000, 8 profile words) fits 1 MB and that minimises the rows per
    cluster ceil(H * S/sq / P) * sq, P = 16 for all clusters, else 1."""
    P = 16 if cluster < 0 else 1
    best, best_rows = 0, 0
    for sq in (S, 256, 128, 64):
        if sq == 0 or sq > S or S % sq or sq % 4:
            continue
        kb, qb, sb = S * dh * 2, sq * dh * 2, sq * S * 2
        if 0x1000 + 2 * qb + 3 * kb + sb + sq * 4 + 32 > 0x100000:
            continue
        rows = -(-H * (S // sq) // P) * sq
        if not best or rows < best_rows:
            best, best_rows = sq, rows
    return best


def main() -> None:
    root = _ref_root()
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "tests" / "gvsoc"))
    from softhier_mlir.testing import lcg, siglip_ref  # noqa: E402
    from softhier_mlir.frontend import siglip  # noqa: E402

    # ---- LCG ------------------------------------------------------------------------------
    out = {}
    for seed, n in [(1, 1), (3, 4095), (3, 4096), (3, 4097), (11, 20000), (0xDEADBEEF, 9000), (0, 70000)]:
        out[f"draws_{seed}_{n}"] = lcg._lcg_stream(seed, n)
    fills = [(64, 96, 7, -16, 16, 0.125), (256, 768, 1, -16, 16, 0.125), (33, 17, 5, -1024, 1023, 1 / 1024),
             (8, 4096, 13, 1, 8, 0.25), (100, 300, 99, -8, 8, 1 / 128), (1, 3072, 12, -4, 4, 0.0625),
             (17, 31, 2, -2, 2, 1.0), (16, 16, 4, 7, 7, 1.0), (40, 40, 21, -60000, 60000, 1.0)]
    for i, (r, c, s, lo, hi, sc) in enumerate(fills):
        out[f"fill_{i}"] = lcg.fill_fp16(r, c, s, lo, hi, sc).view(np.uint16)
        out[f"fill_{i}_args"] = np.array([r, c, s, lo, hi, sc], dtype=np.float64)
    out["const"] = lcg.const_fp16(5, 7, 0x3C00).view(np.uint16)
    out["colparity"] = lcg.col_parity_fp16(4, 9, 15360, 14336).view(np.uint16)
    for seed, r, c, n in [(200, 256, 768, 64), (9, 256, 256, 32), (7, 3, 5, 20)]:
        out[f"samples_{seed}_{r}_{c}_{n}"] = np.array(lcg.sample_positions(r, c, seed, n), dtype=np.int64)
    np.savez_compressed(HERE / "lcg.npz", **out)

    # ---- SigLIP layer, small shapes: every tensor --------------------------------------------
    small = {}
    for S, D, F, H in [(32, 64, 128, 2), (64, 128, 256, 2)]:
        ref = siglip_ref.layer_reference(S, D, F, H)
        for k, v in ref.items():
            small[f"{S}_{D}_{F}_{H}_{k}"] = np.asarray(v, dtype=np.float32)
    np.savez_compressed(HERE / "siglip_small.npz", **small)

    # ---- SigLIP layer S=256: samples at the frontend's dump seeds -----------------------------
    ref = siglip_ref.layer_reference(256, 768, 3072, 12)
    seeds = {"X": 200, "LN1": 206, "Q": 201, "K": 207, "KT": 208, "P0": 209, "V": 211, "O": 202, "H": 203,
             "G": 204, "OUT": 205}
    big = {}
    for tag, seed in seeds.items():
        a = np.asarray(ref[tag], dtype=np.float32)
        pos = np.array(lcg.sample_positions(a.shape[0], a.shape[1], seed, 64), dtype=np.int64)
        big[f"{tag}_pos"] = pos
        big[f"{tag}_val"] = a[pos[:, 0], pos[:, 1]]
        big[f"{tag}_sum"] = np.array([a.astype(np.float64).sum(), np.abs(a.astype(np.float64)).sum()])
    np.savez_compressed(HERE / "siglip_s256.npz", **big)

    # ---- attention_reference (tests/gvsoc/run.py) ----------------------------------------------
    import run  # noqa: E402
    att = {}
    for S, D, H in [(64, 128, 2), (256, 768, 12)]:
        o = run.attention_reference(S, D, H)
        att[f"{S}_{D}_{H}_o"] = o.astype(np.float16).view(np.uint16)
        if S > 64:   # the inputs are LCG fills (pinned by lcg.npz); keep them only for the small case
            continue
        att[f"{S}_{D}_{H}_q"] = lcg.fill_fp16(S, D, 21, -8, 8, 0.125).view(np.uint16)
        att[f"{S}_{D}_{H}_k"] = lcg.fill_fp16(S, D, 22, -8, 8, 0.125).view(np.uint16)
        att[f"{S}_{D}_{H}_v"] = lcg.fill_fp16(S, D, 23, -16, 16, 0.125).view(np.uint16)
    np.savez_compressed(HERE / "attention.npz", **att)

    # ---- Llama-style decoder ops (frontend/smolvla_expert.py numpy twins, frontend/smolvla.py) ---------------
    from softhier_mlir.frontend import smolvla, smolvla_expert as ex  # noqa: E402
    llm = {}
    x = lcg.fill_fp16(64, 192, 31, -64, 64, 1.0 / 32)
    g = lcg.fill_fp16(1, 192, 32, 2, 6, 0.25)
    llm["rms_x"], llm["rms_g"] = x.view(np.uint16), g.view(np.uint16)
    llm["rms_y"] = ex.np_rmsnorm(x, g).astype(np.float16).view(np.uint16)
    xr = lcg.fill_fp16(16, 256, 33, -64, 64, 1.0 / 32)
    tab = smolvla.rope_table(np.arange(16) * 3, 64).astype(np.float16)
    llm["rope_x"], llm["rope_tab"] = xr.view(np.uint16), tab.view(np.uint16)
    llm["rope_y"] = ex.np_rope(xr, tab, 64).astype(np.float16).view(np.uint16)
    ga = lcg.fill_fp16(32, 128, 34, -128, 128, 1.0 / 32)
    ub = lcg.fill_fp16(32, 128, 35, -64, 64, 1.0 / 32)
    llm["silu_a"], llm["silu_b"] = ga.view(np.uint16), ub.view(np.uint16)
    gf, uf = ga.astype(np.float32), ub.astype(np.float32)
    llm["silu_y"] = ex._r16(gf / (1 + np.exp(-gf)) * uf).astype(np.float16).view(np.uint16)   # np_layer's M
    ps = lcg.fill_fp16(64, 32, 36, -100, 100, 1.0 / 64)
    llm["ps_x"] = ps.view(np.uint16)
    llm["ps_y"] = smolvla.pixel_shuffle_gather(ps, 4).view(np.uint16)
    assert np.array_equal(smolvla.pixel_shuffle(ps, 4), smolvla.pixel_shuffle_gather(ps, 4))
    S = 64
    q = lcg.fill_fp16(S, 3 * ex.DH, 37, -32, 32, 1.0 / 32)
    k = lcg.fill_fp16(S, ex.DH, 38, -32, 32, 1.0 / 32)
    v = lcg.fill_fp16(S, ex.DH, 39, -64, 64, 1.0 / 32)
    tok = np.zeros(S, np.uint16)
    tok[[5, 17, 40, 41, 63]] = ex.PAD_TOK
    llm["gqa_q"], llm["gqa_k"], llm["gqa_v"], llm["gqa_tok"] = q.view(np.uint16), k.view(np.uint16), \
        v.view(np.uint16), tok
    llm["gqa_o"] = ex.np_attention(q, k, v, None, None, tok).astype(np.float16).view(np.uint16)
    np.savez_compressed(HERE / "llm.npz", **llm)

    # ---- HBM preload image (softhier_mlir/sim/preload.py) ----------------------------------------------------
    from softhier_mlir.sim import preload  # noqa: E402
    arrays = {0x1000: lcg.fill_fp16(16, 32, 41, -100, 100, 1.0 / 64),
              0x2040: np.arange(100, dtype=np.uint8),
              0x3000: lcg.fill_fp16(8, 64, 42, -8, 8, 0.125)}
    arrays[0x4000] = preload.sentinel_array()
    preload.make_preload_elf(HERE / "preload_small.elf", arrays)
    seg = preload.read_preload_elf(HERE / "preload_small.elf")
    np.savez_compressed(HERE / "preload_small.npz", offsets=np.array(sorted(seg), np.uint64),
                        **{f"seg_{off:x}": np.frombuffer(seg[off], np.uint8) for off in seg})

    # ---- frontend output (dialect text the emitter must lower) ---------------------------------
    mdir = HERE / "mlir"
    mdir.mkdir(exist_ok=True)
    siglip.attention_q_block = _q_block_rule
    # the per-head path hard-codes 256-row GEMM tiles (frontend/siglip.py:126-127), so it needs S % 256 == 0;
    # the small fused case takes explicit 64^3 GEMM tiles, which the library's divisibility check accepts
    cases = {
        "siglip_s256_perhead.mlir": dict(seq=256, d=768, ff=3072, heads=12, fused_attention=False, tiles=None),
        "siglip_s256_fused.mlir": dict(seq=256, d=768, ff=3072, heads=12, fused_attention=True, tiles=None),
        "siglip_s64_fused_l2.mlir": dict(seq=64, d=128, ff=256, heads=2, layers=2, fused_attention=True,
                                         tiles="64,64,64"),
    }
    for name, kw in cases.items():
        text = siglip.emit(cluster=-1, test=True, **kw)
        (mdir / name).write_text(text)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")), sorted(p.name for p in mdir.glob("*.mlir")))


if __name__ == "__main__":
    main()
