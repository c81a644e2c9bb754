"""CPU restatement of native KVarN4 range attention (test infrastructure only).

Follows the reference's descriptor-v1 resident-image contract
(docs/rkva-kvarn-range.md "Descriptor and records"; the reference kernel
shaders/rkva/rkva_range_attn_kvarn4.hlsl:64-150 states the row sources and the
mixed-domain accumulation; its float64 model tests/rkva_range_kvarn4_opt_model.py
oracle_sources/oracle_attention is what the golden fixtures pin this against).

Plane layout (one for K, one for V), head_dim 256 = two 128-wide physical
slices per KV head:
  records  [ceil(capacity / 128) groups][2 * n_head_kv physical heads][8960 B]
           8192 B of 4-bit values, low nibble first, as a 128 x 128 matrix
           (K: [dim][token], V: [token][dim]), then 128 F16 scales and 128 F16
           zero points (per matrix row) and 128 F16 factors (per column);
           value = (q * scale + zero) * factor
  stage    [384 rows = 3 slots x 128][n_head_kv][256] F16, rotated domain;
           global group 0 -> slot 0, global group g > 0 -> slot 1 + (g - 1) % 2
  tail     [128 rows][n_head_kv][256] F16, original domain (precision tail
           length 128; absent when it is 0); row r at r % 128
Row sources for a resident image of `active` rows: rows >= active - tail come
from the tail (original domain); rows of global group 0 and of the incomplete
live group from the stage; the others from the records (rotated domain).
Rotated rows meet the query as WHT256(q) and their value numerator goes back
through WHT256 (Sylvester H256 / 16, symmetric and orthonormal).
"""
from __future__ import annotations

import numpy as np

RECORD = 8960
GROUP = 128
STAGE_ROWS = 384
D = 256


class Desc:
    def __init__(self, origin: int, capacity: int, tail: int, n_head_kv: int):
        assert origin % GROUP == 0 and tail in (0, GROUP)
        self.origin, self.capacity, self.tail, self.n_head_kv = origin, capacity, tail, n_head_kv
        self.groups = (capacity + GROUP - 1) // GROUP
        self.phys = 2 * n_head_kv
        self.records_bytes = self.groups * self.phys * RECORD
        self.row_bytes = n_head_kv * D * 2
        self.stage_bytes = STAGE_ROWS * self.row_bytes
        self.plane_bytes = self.records_bytes + self.stage_bytes + (GROUP * self.row_bytes
                                                                    if tail else 0)


def stage_slot(global_group: int) -> int:
    return 0 if global_group == 0 else 1 + (global_group - 1) % 2


def staged(desc: Desc, group: int, active: int) -> bool:
    live = (active - 1) // GROUP if active else 0
    return desc.origin // GROUP + group == 0 or (group == live and active % GROUP != 0)


def make_plane(desc: Desc, active: int, seed: int) -> np.ndarray:
    """A seeded plane: records for every complete group, stage rows for the
    staged groups, tail rows for the last min(active, tail) rows; everything
    else 0xFF bytes (F16 NaN) so that a stray read shows."""
    rng = np.random.default_rng(seed)
    buf = np.full(desc.plane_bytes, 0xFF, np.uint8)
    for g in range(active // GROUP):
        for ph in range(desc.phys):
            off = (g * desc.phys + ph) * RECORD
            buf[off:off + 8192] = rng.integers(0, 256, 8192, dtype=np.uint8)
            scale = rng.uniform(0.01, 0.12, GROUP) * rng.choice([-1.0, 1.0], GROUP)
            zero = rng.uniform(-0.5, 0.5, GROUP)
            other = rng.uniform(0.5, 1.5, GROUP) * rng.choice([-1.0, 1.0], GROUP)
            axes = np.concatenate([scale, zero, other]).astype("<f2")
            buf[off + 8192:off + RECORD] = axes.view(np.uint8)
    groups = {(active - 1) // GROUP} if active % GROUP else set()
    if desc.origin == 0 and active:
        groups.add(0)
    for g in sorted(groups):
        rows = GROUP if (g + 1) * GROUP <= active else active - g * GROUP
        slot = stage_slot(desc.origin // GROUP + g)
        vals = (rng.normal(0, 0.5, rows * desc.n_head_kv * D)).astype("<f2")
        off = desc.records_bytes + slot * GROUP * desc.row_bytes
        buf[off:off + vals.nbytes] = vals.view(np.uint8)
    if desc.tail:
        for r in range(active - min(active, desc.tail), active):
            vals = rng.normal(0, 0.5, desc.n_head_kv * D).astype("<f2")
            off = desc.records_bytes + desc.stage_bytes + (r % GROUP) * desc.row_bytes
            buf[off:off + desc.row_bytes] = vals.view(np.uint8)
    return buf


def decode_record(blob: np.ndarray, value: bool) -> np.ndarray:
    """[token][dim] float32 of one record (K is stored [dim][token])."""
    nib = np.empty(GROUP * GROUP, np.float32)
    nib[0::2] = blob[:8192] & 15
    nib[1::2] = blob[:8192] >> 4
    m = nib.reshape(GROUP, GROUP)                 # [row][col]
    axes = blob[8192:RECORD].view("<f2").astype(np.float32).reshape(3, GROUP)
    with np.errstate(over="ignore", invalid="ignore"):
        affine = (m * axes[0][:, None]).astype(np.float32) + axes[1][:, None]
        x = (affine.astype(np.float32) * axes[2][None, :]).astype(np.float32)
    return x if value else x.T


def sources(desc: Desc, plane: np.ndarray, active: int, value: bool):
    """[active][n_head_kv][256] float32 in each row's storage domain, and the
    mask of original-domain (tail) rows."""
    out = np.zeros((active, desc.n_head_kv, D), np.float32)
    tail_begin = active - min(active, desc.tail)
    stage = plane[desc.records_bytes:desc.records_bytes + desc.stage_bytes].view("<f2")
    stage = stage.astype(np.float32).reshape(STAGE_ROWS, desc.n_head_kv, D)
    tail = None
    if desc.tail:
        t0 = desc.records_bytes + desc.stage_bytes
        tail = plane[t0:t0 + GROUP * desc.row_bytes].view("<f2").astype(np.float32)
        tail = tail.reshape(GROUP, desc.n_head_kv, D)
    cache = {}
    for r in range(active):
        g, pos = divmod(r, GROUP)
        if r >= tail_begin:
            out[r] = tail[r % GROUP]
        elif staged(desc, g, active):
            out[r] = stage[stage_slot(desc.origin // GROUP + g) * GROUP + pos]
        else:
            for kv in range(desc.n_head_kv):
                for s in range(2):
                    key = (g, 2 * kv + s)
                    if key not in cache:
                        off = (g * desc.phys + 2 * kv + s) * RECORD
                        cache[key] = decode_record(plane[off:off + RECORD], value)
                    out[r, kv, s * GROUP:(s + 1) * GROUP] = cache[key][pos]
    return out, np.arange(active) >= tail_begin


def hadamard256() -> np.ndarray:
    h = np.array([[1.0]])
    for _ in range(8):
        h = np.block([[h, h], [h, -h]])
    return h / 16.0


def attend(desc: Desc, k_plane, v_plane, active: int, q, positions, scale: float,
           n_head: int):
    """float64 attention in the original domain.  q [n_tokens][n_head][256];
    returns out [n_tokens][n_head][256], lse [n_tokens][n_head] (natural log;
    empty rows: 0 and -inf)."""
    H = hadamard256()
    k, exact = sources(desc, k_plane, active, False)
    v, _ = sources(desc, v_plane, active, True)
    k = k.astype(np.float64)
    v = v.astype(np.float64)
    body = ~exact
    k[body] = k[body] @ H
    v[body] = v[body] @ H
    nt = len(positions)
    out = np.zeros((nt, n_head, D))
    lse = np.full((nt, n_head), -np.inf)
    g = n_head // desc.n_head_kv
    for t in range(nt):
        pos = int(positions[t])
        limit = 0 if pos < desc.origin else min(active, pos - desc.origin + 1)
        if limit == 0:
            continue
        for h in range(n_head):
            kv = h // g
            s = (k[:limit, kv] @ q[t, h].astype(np.float64)) * scale
            mx = s.max()
            w = np.exp(s - mx)
            out[t, h] = (w @ v[:limit, kv]) / w.sum()
            lse[t, h] = mx + np.log(w.sum())
    return out, lse
