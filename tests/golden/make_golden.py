"""Generates tests/golden/q8_golden.npz from the REFERENCE ITSELF (oracle/_ref/libllama_ref.so, compiled from
LucianCrainic/llama3.x.c's own sources by oracle/Makefile), on seeded inputs.

    make -C oracle REF=REFERENCE_CHECKOUT && python tests/golden/make_golden.py

Cases (all small; numpy PCG64 seeds below):
  quant_ties      k_quantize on the reference test suite's tie values at scale 1 (tests/kernels.c:111-116: 127, 2.5,
                  -3.5, 0.5, -0.5, 1.5, -126.5, 0, then zeros and an all-zero group), gs 16, n 64
  quant_<n>_<gs>  k_quantize, scalar and AVX-512 ISAs (bitwise equal), N(0,1) inputs
  gemv_*          k_matmul_q8 on the scalar ISA (q8_dots, src/gemv.c:417-438)
  amx_*           k_gemm_q8 on the AMX-INT8 backend (amx_q8_chunk, src/gemm.c:554-610) + its exact int32 group dots
                  (k_gemm_q8_amx_dots_test)
  rms_*           k_rmsnorm on the AVX-512 ISA (src/kernels_simd.c:136-161) and the scalar one (src/kernels.c:8-21)
  gemvf_*         k_matmul_q8 on fp32 activations (W8A32), AVX-512 ISA for gs % 16 == 0, else scalar
  gemv512_*       k_matmul_q8 on the AVX-512 ISA (dots_q8_body, src/gemv.c:109-139), the reference's decode GEMV
  vnni_*          pack_s8_vnni of a 37 x 200 slice (row stride 256)
"""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import oracle as O  # noqa: E402


def main():
    if not O.ref_available():
        raise SystemExit("oracle/_ref/libllama_ref.so is missing: run `make -C oracle REF=<reference checkout>`")
    rng = np.random.default_rng(20261201)
    out = {}
    ties = np.zeros(64, np.float32)
    ties[:8] = [127, 2.5, -3.5, 0.5, -0.5, 1.5, -126.5, 0]
    ties[32:] = rng.standard_normal(32).astype(np.float32) * 3
    q, s = O.ref_quantize(ties, 16, O.KERNELS_SCALAR)
    out.update(quant_ties_x=ties, quant_ties_gs=np.int32(16), quant_ties_q=q, quant_ties_s=s)
    for n, gs in [(256, 64), (4096, 64), (512, 128), (192, 32), (1792, 64)]:
        x = (rng.standard_normal(n) * rng.uniform(0.01, 10)).astype(np.float32)
        q, s = O.ref_quantize(x, gs, O.KERNELS_AVX512)
        q2, s2 = O.ref_quantize(x, gs, O.KERNELS_SCALAR)
        assert (q == q2).all() and (s.view(np.int32) == s2.view(np.int32)).all()
        out.update({f"quant_{n}_{gs}_x": x, f"quant_{n}_{gs}_q": q, f"quant_{n}_{gs}_s": s})
    for d, n in [(37, 1024), (16, 4096)]:
        wq, ws = O.seeded_q8_matrix(d, n, 64, seed=d)
        xq, xs = O.quantize(rng.standard_normal(n).astype(np.float32), 64)
        out.update({f"gemv_{d}_{n}_wq": wq, f"gemv_{d}_{n}_ws": ws, f"gemv_{d}_{n}_xq": xq, f"gemv_{d}_{n}_xs": xs,
                    f"gemv_{d}_{n}_y": O.ref_gemv(xq, xs, wq, ws, 64, O.KERNELS_SCALAR)})
    if O.ref_amx_unavailable() is None:
        for m, d, k in [(1, 40, 512), (7, 48, 1024), (33, 32, 256)]:
            wq, ws = O.seeded_q8_matrix(d, k, 64, seed=100 + m)
            xq, xs = O.quantize(rng.standard_normal((m, k)).astype(np.float32), 64)
            c = O.ref_gemm_amx(xq, xs, wq, ws, 64)
            L = O.ref()
            import ctypes
            packed = np.zeros(L.s8_vnni_bytes(d, k), np.int8)
            L.pack_s8_vnni(O._p(packed, O._i8p), O._p(wq, O._i8p), d, k, k)
            pad = np.zeros(((m + 31) // 32 * 32, k), np.int8)
            pad[:m] = xq
            dots = np.zeros((k // 64, m, d), np.int32)
            assert O.ref_select(O.KERNELS_AMX)
            assert L.k_gemm_q8_amx_dots_test(O._p(dots, O._i32p), O._p(pad, O._i8p), m, k, 64,
                                             O._p(packed, O._i8p), d)
            O.ref_select(O.KERNELS_SCALAR)
            key = f"amx_{m}_{d}_{k}"
            out.update({key + "_wq": wq, key + "_ws": ws, key + "_xq": xq, key + "_xs": xs, key + "_c": c,
                        key + "_dots": dots})
    for n in [17, 64, 2048, 4099]:
        x = rng.standard_normal(n).astype(np.float32)
        w = rng.uniform(0.5, 1.5, n).astype(np.float32)
        out.update({f"rms_{n}_x": x, f"rms_{n}_w": w,
                    f"rms_{n}_avx512": O.ref_rmsnorm(x, w, 1e-5, O.KERNELS_AVX512),
                    f"rms_{n}_scalar": O.ref_rmsnorm(x, w, 1e-5, O.KERNELS_SCALAR)})
    # W8A32 (fp32 activations, K8Input.q NULL): k_matmul_q8 on the AVX-512 ISA (dots_q8f_body, src/gemv.c:141-180)
    # for gs % 16 == 0, else the portable loop (src/gemv.c:427-436).
    for d, n, gs in [(37, 1024, 64), (16, 512, 32), (20, 256, 16), (9, 384, 128), (8, 96, 48), (6, 40, 2)]:
        wq, ws = O.seeded_q8_matrix(d, n, gs, seed=d + n)
        x = (rng.standard_normal(n) * rng.uniform(0.1, 5)).astype(np.float32)
        isa = O.KERNELS_AVX512 if gs % 16 == 0 else O.KERNELS_SCALAR
        key = f"gemvf_{d}_{n}_{gs}"
        out.update({key + "_wq": wq, key + "_ws": ws, key + "_x": x, key + "_y": O.ref_gemv_f32(x, wq, ws, gs, isa)})
    # The reference's AMX int8 packing (pack_s8_vnni, src/gemm.c:384-398) of a ragged matrix with a row stride.
    L = O.ref()
    w = rng.integers(-127, 128, size=(37, 256), dtype=np.int8)
    packed = np.zeros(L.s8_vnni_bytes(37, 200), np.int8)
    L.pack_s8_vnni(O._p(packed, O._i8p), O._p(w, O._i8p), 37, 200, 256)
    out.update(vnni_w=w, vnni_packed=packed)
    # The reference's decode GEMV on an AVX-512 host (generated last, so the arrays above keep their values).
    for d, n, gs in [(37, 1024, 64), (16, 4096, 64), (9, 512, 128), (5, 768, 256), (8, 14336, 64)]:
        wq, ws = O.seeded_q8_matrix(d, n, gs, seed=7 * d + n)
        xq, xs = O.quantize((rng.standard_normal(n) * rng.uniform(0.1, 5)).astype(np.float32), gs)
        key = f"gemv512_{d}_{n}_{gs}"
        out.update({key + "_wq": wq, key + "_ws": ws, key + "_xq": xq, key + "_xs": xs,
                    key + "_y": O.ref_gemv(xq, xs, wq, ws, gs, O.KERNELS_AVX512)})
    path = Path(__file__).with_name("q8_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({path.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
