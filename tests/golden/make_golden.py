#!/usr/bin/env python3
"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run here, where the reference checkout exists (it does not on the GPU box):

    make -C oracle ref            # compiles oracle/_ref/libxq_gdn_ref.so
    python tests/golden/make_golden.py [--reference DIR]   # default: $XQ_REFERENCE

Sources of truth (none of them this repository's own code):
  codecs.npz      gguf 0.19.0 gguf/quants.py Q8_0 / Q4_0 quantize + dequantize
                  (bit-exact with ggml-quants.c), numpy float16 casts (RNE).
  range_*.npz     the reference's own CPU models of its decode kernels:
                  tests/rkva_range_q4_opt_model.py (float64 oracle(),
                  run_reference_exact(): rkva_range_attn.hlsl +
                  rkva_range_reduce.hlsl in float32) and
                  tests/rkva_range_fmt_opt_model.py (make_rows /
                  independent_decode for F16 and Q8_0 records).
  reduce.npz      tests/rkva_range_kvarn4_opt_model.py reduce_partials() on
                  the empty / poisoned / overflow states of
                  tests/rkva_range_reduce_finite_model.py.
  kvarn4.npz      tests/rkva_range_kvarn4_opt_model.py oracle_sources() +
                  oracle_attention() (float64, explicit Sylvester H256/16) on
                  planes built by oracle/kvarn4.make_plane from the stored
                  seeds (with each plane's SHA-256 to catch drift).
  gdn_selftest.npz  src/bridge/ggml_d3d12.cpp:113-158 d3d12_gdn_emulate
                  (compiled by oracle/build_ref.sh) on the selftest protocol
                  of ggml_d3d12.cpp:174-369, plus the first draws of
                  libstdc++ std::mt19937 / uniform_real_distribution<float>.
"""
import argparse
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)


def make_codecs(out):
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as QT

    rng = np.random.default_rng(20261201)
    x = rng.normal(0, 1, (64, 256)).astype(np.float32)
    edge = np.zeros((8, 256), np.float32)
    edge[1, 5] = 3.0                      # single nonzero
    edge[2, :32] = -np.arange(32)         # negative extreme
    edge[3, :32] = np.linspace(-1, 1, 32)
    edge[4, :64] = rng.normal(0, 1e-6, 64)  # tiny scale (f16 subnormal d)
    edge[5, :32] = 65504.0 / 2            # large
    edge[6, :32] = 127.0 * (np.arange(32) % 2 * 2 - 1) + 0.5  # round-half cases
    edge[7, :32] = np.arange(32) - 16.0 + 0.5
    x = np.concatenate([x, edge])
    q8 = quants.quantize(x, QT.Q8_0)
    q4 = quants.quantize(x, QT.Q4_0)
    np.savez_compressed(
        os.path.join(out, "codecs.npz"), x=x, q8=q8, q8_deq=quants.dequantize(q8, QT.Q8_0),
        q4=q4, q4_deq=quants.dequantize(q4, QT.Q4_0),
        f16_in=np.concatenate([x[:4].ravel(), np.array(
            [0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e-8, 2.0 ** -25, 2.0 ** -24 * 1.5,
             6.1e-5, -3.0e-7, np.inf, -np.inf], np.float32)]).astype(np.float32))
    d = np.load(os.path.join(out, "codecs.npz"))
    np.savez_compressed(os.path.join(out, "codecs.npz"), **{k: d[k] for k in d.files},
                        f16_bits=d["f16_in"].astype(np.float16).view(np.uint16))


def make_range(out, ref_tests):
    sys.path.insert(0, ref_tests)
    import rkva_range_fmt_opt_model as mf
    import rkva_range_q4_opt_model as m4

    rng = np.random.default_rng(20261202)
    scale = np.float32(1.0 / 16.0)
    origin = 102400
    cases = [(1, 0), (40, 39), (64, 19), (48, -5), (300, 299)]
    for storage, name in ((0, "f16"), (2, "q8_0"), (1, "q4_0")):
        arrays = {}
        for ci, (active, rel) in enumerate(cases):
            if storage != 1 and active > 64:
                continue  # keep F16/Q8_0 fixtures small; Q4_0 covers 2 splits
            rows = max(active, 1)
            if storage == 1:
                kb, vb = m4.make_q4_rows(rng, rows), m4.make_q4_rows(rng, rows)
                k, v = m4.dequant_table(kb, rows), m4.dequant_table(vb, rows)
            else:
                kb, vb = mf.make_rows(storage, rng, rows), mf.make_rows(storage, rng, rows)
                k = mf.independent_decode(storage, kb, rows)
                v = mf.independent_decode(storage, vb, rows)
            q = rng.normal(0, 2, (m4.N_HEAD, m4.D)).astype(np.float32)
            pos = origin + rel
            causal = 0 if pos < origin else pos - origin + 1
            limit = min(active, causal)
            o64, l64 = m4.oracle(q, k, v, limit, scale)
            r_out, r_lse = m4.run_reference_exact(q, k, v, active, limit, scale)
            arrays.update({
                f"c{ci}_k": np.frombuffer(kb, np.uint8), f"c{ci}_v": np.frombuffer(vb, np.uint8),
                f"c{ci}_q": q,
                f"c{ci}_meta": np.array([active, pos, origin, limit, m4.reference_split_k(active)],
                                        np.int64),
                f"c{ci}_o64": o64.astype(np.float64), f"c{ci}_l64": l64.astype(np.float64),
                f"c{ci}_oref": r_out, f"c{ci}_lref": r_lse})
        arrays["shape"] = np.array([m4.N_HEAD, m4.N_HEAD_KV, m4.D], np.int64)
        np.savez_compressed(os.path.join(out, f"range_{name}.npz"), **arrays)
    # split policy table (rkva-range-profile.h via the q4 model's restatement)
    actives = np.array([0, 1, 31, 32, 33, 127, 128, 129, 255, 256, 257, 1000, 4096, 8192, 8193,
                        16384, 32768, 65536, 262144], np.int64)
    pol = np.array([[m4.reference_split_k(a)] + [m4.optimized_split_k(a, m) for m in (1, 2, 3)]
                    for a in actives], np.int64)
    np.savez_compressed(os.path.join(out, "split_policy.npz"), active=actives, split_k=pol)


def make_reduce(out, ref_tests):
    sys.path.insert(0, ref_tests)
    import rkva_range_kvarn4_opt_model as model

    def st(maximum=0.0, den=1.0, num=2.0):
        return (np.array([maximum], np.float32), np.array([den], np.float32),
                np.full((1, 256), num, np.float32))

    huge = np.finfo(np.float32).max
    empty = st(-np.inf, 0.0, np.nan)
    bad_num = st(-1000.0)
    bad_num[2][0, 173] = np.nan
    rng = np.random.default_rng(20261203)
    rand = [(rng.normal(0, 3, 1).astype(np.float32), rng.uniform(0.5, 40, 1).astype(np.float32),
             rng.normal(0, 1, (1, 256)).astype(np.float32)) for _ in range(7)]
    cases = {
        "all_empty": [empty] * 5,
        "empty_then_valid": [empty] * 3 + [st()],
        "bad_den_nan": [st(), st(den=np.nan)],
        "bad_den_neg": [st(den=-1.0), st()],
        "bad_max_inf": [st(), st(maximum=np.inf)],
        "bad_num_under_zero_weight": [st(), bad_num],
        "den_overflow": [st(den=huge)] * 2,
        "num_overflow": [st(num=huge)] * 2,
        "random7": rand,
    }
    arrays = {}
    for name, states in cases.items():
        o, l = model.reduce_partials(states, rotated=False)
        parts = np.stack([np.concatenate([a[0], s[0], s[1]]) for s in states
                          for a in [s[2]]])[:, None, :]
        arrays[f"{name}_partials"] = parts.astype(np.float32)
        arrays[f"{name}_out"] = o
        arrays[f"{name}_lse"] = l
    np.savez_compressed(os.path.join(out, "reduce.npz"), **arrays)


def make_gdn(out):
    import oracle

    ref = oracle.ref_gdn_lib()
    if ref is None:
        raise SystemExit("oracle/_ref/libxq_gdn_ref.so missing: run `make -C oracle ref`")
    arrays = {}
    draws = np.empty((6, 64), np.float32)
    for j in range(6):
        ref.xq_std_uniform(1701 + j, -0.05, 0.05, 64, draws[j].ctypes.data)
    arrays["std_uniform_1701_1706"] = draws
    cases = [(5, 5, 0), (1, 5, 0), (2, 5, 0), (3, 5, 0), (4, 5, 0), (64, 5, 0), (5, 1, 0),
             (1, 1, 0), (64, 1, 0), (3, 5, 3), (4, 5, 3)]
    sample_idx = np.arange(0, 524288, 257)
    for T, K, pad in cases:
        n = 4096 * T + 524288 * K
        o = np.full(n, 1e30, np.float32)
        rc = ref.xq_gdn_ref_run(T, K, pad, None, None, None, None, None, None, o.ctypes.data)
        assert rc == 0, (T, K, pad)
        key = f"T{T}_K{K}_p{pad}"
        y = o[:4096 * T].reshape(T, 32, 128)
        arrays[key + "_y_head"] = y[:min(T, 5)]
        arrays[key + "_y_sum"] = y.astype(np.float64).sum(axis=2)
        snaps = o[4096 * T:].reshape(K, 32, 128 * 128)
        written = min(T, K)
        arrays[key + "_snap_sum"] = snaps[:written].astype(np.float64).sum(axis=2)
        arrays[key + "_snap_sq"] = (snaps[:written].astype(np.float64) ** 2).sum(axis=2)
        arrays[key + "_snap_sample"] = snaps[:written].reshape(written, -1)[:, sample_idx]
        arrays[key + "_unwritten_all_sentinel"] = np.array(
            [bool(np.all(snaps[written:] == np.float32(1e30)))])
    arrays["snap_sample_idx"] = sample_idx
    np.savez_compressed(os.path.join(out, "gdn_selftest.npz"), **arrays)


# (origin, capacity, precision tail, active, positions relative to origin, seed)
KVARN4_CASES = [
    (0, 640, 0, 520, [519], 11),
    (0, 640, 128, 520, [300], 12),
    (102400, 4224, 128, 4133, [4132, 4000], 13),
    (128, 512, 128, 512, [511, -5, 200], 14),
    (256, 1024, 0, 1000, [999], 15),
]


def make_kvarn4(out, ref_tests):
    import hashlib
    sys.path.insert(0, ref_tests)
    import rkva_range_kvarn4_opt_model as km
    from oracle import kvarn4 as ok
    arrays = {}
    for i, (origin, cap, tail, active, rel, seed) in enumerate(KVARN4_CASES):
        desc = ok.Desc(origin, cap, tail, km.N_HEAD_KV)
        lay = km.Layout(origin, cap, tail)
        assert lay.half == desc.plane_bytes
        kp = ok.make_plane(desc, active, seed)
        vp = ok.make_plane(desc, active, seed + 1000)
        rng = np.random.default_rng(seed + 2000)
        q = rng.normal(0, 1, (len(rel), km.N_HEAD, km.D)).astype(np.float32)
        pos = np.array([origin + r for r in rel], np.int32)
        ks, exact = km.oracle_sources(lay, kp.tobytes(), active, False)
        vs, _ = km.oracle_sources(lay, vp.tobytes(), active, True)
        outs, lses = [], []
        for t, p in enumerate(pos):
            limit = km.causal_limit(lay, active, int(p))
            o, l = km.oracle_attention(q[t], ks, vs, exact, limit, 1 / 16.0)
            outs.append(o)
            lses.append(l)
        key = "c%d" % i
        arrays[key + "_cfg"] = np.array([origin, cap, tail, active, seed], np.int64)
        arrays[key + "_pos"] = pos
        arrays[key + "_q"] = q
        arrays[key + "_out"] = np.array(outs)
        arrays[key + "_lse"] = np.array(lses)
        arrays[key + "_sha"] = np.frombuffer(
            hashlib.sha256(kp.tobytes() + vp.tobytes()).digest(), np.uint8)
    np.savez_compressed(os.path.join(out, "kvarn4.npz"), **arrays)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get(
        "XQ_REFERENCE", os.path.join(os.path.dirname(REPO), "reference")))
    ap.add_argument("--only", default=None, help="codecs|range|reduce|kvarn4|gdn")
    args = ap.parse_args()
    ref_tests = os.path.join(args.reference, "tests")
    steps = {"codecs": lambda: make_codecs(HERE), "range": lambda: make_range(HERE, ref_tests),
             "reduce": lambda: make_reduce(HERE, ref_tests),
             "kvarn4": lambda: make_kvarn4(HERE, ref_tests), "gdn": lambda: make_gdn(HERE)}
    for name, fn in steps.items():
        if args.only in (None, name):
            fn()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
