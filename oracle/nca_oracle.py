"""CPU oracle of the NCA test-time rollout -- TEST INFRASTRUCTURE, NOT PART OF THE PRODUCT.

A plain numpy (fp32) restatement of the reference's algorithm for the rollout path of
JorisViaudQuantAI/NCAs, used only by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline as the checker.  The product (ncas_b200) never imports this module.

Pinning: tests/test_oracle.py checks every function here against golden vectors produced by the
live reference (tests/golden/make_golden.py imports the reference's own nca package and records
its outputs), so the restatement is tied to the reference, not to this file's reading of it.

Each function names the reference code it restates (paths relative to the reference root).
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


# ---------------------------------------------------------------------------- the cell rule
def perceive_nhwc(x: np.ndarray, taps: np.ndarray, pad=None) -> np.ndarray:
    """KernelPerception on a channels-last state: x (B, H, W, C) -> z (B, H, W, heads*C),
    head-major z[..., k*C + c] = sum_n taps[k, n] * x[shifted n, c] (src/nca/model.py:175-178;
    taps summed in row-major order n = 0..8).  The border is zero, or the vector `pad` (C,) for
    wall padding (src/nca/model.py:140-152)."""
    B, H, W, C = x.shape
    heads = taps.shape[0]
    t = taps.reshape(heads, 9).astype(F32)
    xp = np.zeros((B, H + 2, W + 2, C), F32)
    if pad is not None:
        xp[:] = np.asarray(pad, F32)
    xp[:, 1:-1, 1:-1] = x
    z = np.zeros((B, H, W, heads, C), F32)
    tmp = np.empty((B, H, W, C), F32)
    for n in range(9):
        dy, dx = divmod(n, 3)
        v = xp[:, dy : dy + H, dx : dx + W]
        for k in range(heads):
            if t[k, n] != 0:
                np.multiply(v, t[k, n], out=tmp)
                np.add(z[..., k, :], tmp, out=z[..., k, :])
    return z.reshape(B, H, W, heads * C)


def perceive(x: np.ndarray, taps: np.ndarray, pad=None) -> np.ndarray:
    """perceive_nhwc on the reference's (B, C, H, W) layout: z (B, heads*C, H, W)."""
    z = perceive_nhwc(np.ascontiguousarray(x.transpose(0, 2, 3, 1)), taps, pad)
    return np.ascontiguousarray(z.transpose(0, 3, 1, 2))


def mlp_rows(z: np.ndarray, w1, b1, w2, b2) -> np.ndarray:
    """MLPUpdate (src/nca/model.py:277-287) on rows of cells: z (M, P) -> dx (M, C) with
    dx = W2 relu(W1 z + b1) + b2 in fp32."""
    h = z @ w1.reshape(w1.shape[0], -1).T.astype(F32)
    np.add(h, b1.astype(F32), out=h)
    np.maximum(h, F32(0), out=h)
    dx = h @ w2.reshape(w2.shape[0], -1).T.astype(F32)
    np.add(dx, b2.astype(F32), out=dx)
    return dx


def mlp(z: np.ndarray, w1, b1, w2, b2) -> np.ndarray:
    """mlp_rows on the (B, P, H, W) layout."""
    B, P, H, W = z.shape
    dx = mlp_rows(np.ascontiguousarray(z.transpose(0, 2, 3, 1)).reshape(-1, P), w1, b1, w2, b2)
    return np.ascontiguousarray(dx.reshape(B, H, W, -1).transpose(0, 3, 1, 2))


def apply_clamp(x, given4, clamp, in_off: int) -> np.ndarray:
    """NCA.apply_clamp (src/nca/model.py:430-438): input slice of given cells <- clamp."""
    c_in = clamp.shape[1]
    out = x.copy()
    sl = slice(in_off, in_off + c_in)
    out[:, sl] = np.where(given4, clamp, x[:, sl])
    return out


def step_nhwc(x, given, clamp_nhwc, fire, p: dict, noise=None) -> np.ndarray:
    """NCA.step without norm/clock (src/nca/model.py:503-525, residual_update 527-559) on
    channels-last arrays: x (B, H, W, C), given (B, H, W) bool, clamp (B, H, W, c_in),
    fire (B, H, W) {0, 1}, noise (B, H, W, C) or None.  x' = x + fire * dx (+ noise), then the
    clamp."""
    B, H, W, C = x.shape
    z = perceive_nhwc(x, p["taps"], p.get("pad"))
    dx = mlp_rows(z.reshape(B * H * W, -1), p["w1"], p["b1"], p["w2"], p["b2"]).reshape(B, H, W, C)
    np.multiply(dx, fire.reshape(B, H, W, 1).astype(F32), out=dx)
    np.add(dx, x, out=dx)
    if noise is not None:
        np.add(dx, noise, out=dx)
    sl = slice(p["in_off"], p["in_off"] + clamp_nhwc.shape[-1])
    dx[..., sl] = np.where(given[..., None], clamp_nhwc, dx[..., sl])
    return dx


def step(x, given4, clamp, fire, p: dict) -> np.ndarray:
    """step_nhwc on the reference's layouts: x (B, C, H, W), given4 (B, 1, H, W), clamp
    (B, c_in, H, W), fire (B, 1, H, W)."""
    y = step_nhwc(np.ascontiguousarray(x.transpose(0, 2, 3, 1)), given4[:, 0],
                  np.ascontiguousarray(clamp.transpose(0, 2, 3, 1)), np.asarray(fire)[:, 0], p)
    return np.ascontiguousarray(y.transpose(0, 3, 1, 2))


def scores(x, p: dict) -> np.ndarray:
    """Head scores on the readout slice (src/nca/model.py:596-609): (B, n_out, H, W).  'mlp':
    head_w o + head_b; 'l2': 1 / (1 + sqrt(|o - e_v|^2 + 1e-8)) with e_v the output-token
    embeddings (out_embed)."""
    o = x[:, p["out_off"] : p["out_off"] + p["c_out"]]
    if p.get("head", "mlp") == "l2":
        e = np.asarray(p["out_embed"], F32)
        d = o[:, None] - e[None, :, :, None, None]
        return (F32(1) / (F32(1) + np.sqrt((d * d).sum(axis=2) + F32(1e-8)))).astype(F32)
    hw = p["head_w"].reshape(p["head_w"].shape[0], -1).astype(F32)
    return np.einsum("vc,bchw->bvhw", hw, o).astype(F32) + p["head_b"].astype(F32)[None, :, None, None]


def decode(x, p: dict) -> np.ndarray:
    """Argmax token per cell (src/nca/model.py:615-622); first maximum wins."""
    return np.asarray(p["out_tokens"])[scores(x, p).argmax(axis=1)]


def confidence(x, p: dict) -> np.ndarray:
    """Max softmax probability per cell ('mlp' head) or best score ('l2'), clamped to [0, 1]
    (src/nca/model.py:624-629)."""
    s = scores(x, p)
    if p.get("head", "mlp") == "l2":
        return np.clip(s.max(axis=1), 0.0, 1.0).astype(F32)
    m = s.max(axis=1, keepdims=True)
    e = np.exp(s - m)
    return np.clip((e / e.sum(axis=1, keepdims=True)).max(axis=1), 0.0, 1.0).astype(F32)


def board_confidence(x, p: dict) -> np.ndarray:
    """Mean cell confidence over all H*W cells (src/nca/model.py:631-633)."""
    return confidence(x, p).mean(axis=(1, 2), dtype=np.float64).astype(F32)


def decode_boards(x, given, inputs, p: dict) -> np.ndarray:
    """Given cells show their input token (src/nca/rollout.py:74-82)."""
    return np.where(given, inputs, decode(x, p))


def init_state(inputs, given, p: dict, channels: int):
    """sigma_init = 0 state with the input slice of given cells clamped (src/nca/model.py:
    384-412): returns (x, given4, clamp)."""
    B, H, W = inputs.shape
    clamp = np.ascontiguousarray(p["embed"][inputs].transpose(0, 3, 1, 2)).astype(F32)
    given4 = given[:, None]
    x = apply_clamp(np.zeros((B, channels, H, W), F32), given4, clamp, p["in_off"])
    return x, given4, clamp


# ----------------------------------------------------------------------- selection, pruning
def conf_at_k(metric, conf, alive, ks):
    """src/nca/rollout.py:317-334 (unweighted)."""
    N, K = metric.shape
    out = {}
    for k in ks:
        k = min(k, K)
        c = np.where(alive[:, :k], conf[:, :k], -np.inf)
        out[k] = float(np.mean(metric[np.arange(N), c.argmax(axis=1)]))
    return out


def best_trial(conf, alive, k):
    """Per board the first index of the largest alive confidence among trials < k."""
    return np.where(alive[:, :k], conf[:, :k], -np.inf).argmax(axis=1)


def pass_at_k(metric, alive, ks):
    """src/nca/rollout.py:337-350 (unweighted)."""
    N, K = metric.shape
    return {min(k, K): float(np.mean((metric[:, : min(k, K)] & alive[:, : min(k, K)]).any(axis=1)))
            for k in ks}


def niche_capped_pruning(decoded, conf, alive, n_cap, order_fn):
    """The reference's halving rule, src/nca/pruning.py:22-65: niches by decoded-grid bytes,
    at most n_cap per niche (stable sort by -conf), survivors round-robin over niches in the
    order order_fn(n_niches) (the reference draws rng.permutation), until half the alive
    trials are kept.  decoded (N, K, ...) ints, conf (N, K), alive (N, K) bool."""
    N, K = conf.shape
    al = alive.copy()
    for n in range(N):
        idx = np.nonzero(al[n])[0]
        if len(idx) <= 1:
            continue
        target = len(idx) // 2
        niches: dict[bytes, list[int]] = {}
        for k in idx:
            niches.setdefault(np.ascontiguousarray(decoded[n, k]).tobytes(), []).append(int(k))
        capped = [sorted(m, key=lambda k: -conf[n, k])[:n_cap] for m in niches.values()]
        order = order_fn(len(capped))
        surv: list[int] = []
        depth = 0
        while len(surv) < target:
            added = False
            for j in order:
                if depth < len(capped[j]):
                    surv.append(capped[j][depth])
                    added = True
                    if len(surv) >= target:
                        break
            if not added:
                break
            depth += 1
        new = np.zeros(K, dtype=bool)
        new[surv] = True
        al[n] = new
    return al


def niche_cap_refill(decoded, conf, n_cap):
    """Niche-capped pruning with refill (the benchmark's variant of src/nca/pruning.py:22-65):
    niches by identical decoded grid (pruning.py:39-41), the n_cap most confident members of
    each kept (stable sort by -conf, pruning.py:43-46), and every dropped slot, in increasing
    trial order, refilled with a clone of the kept trials ranked by confidence (ties: lower
    trial first), cycling.  Returns (src (N, K) int: slot k continues from trial src[k],
    kept (N, K) bool)."""
    N, K = conf.shape
    src = np.tile(np.arange(K), (N, 1))
    kept = np.zeros((N, K), dtype=bool)
    for n in range(N):
        niches: dict[bytes, list[int]] = {}
        for k in range(K):
            niches.setdefault(np.ascontiguousarray(decoded[n, k]).tobytes(), []).append(k)
        for members in niches.values():
            for k in sorted(members, key=lambda k: -conf[n, k])[:n_cap]:
                kept[n, k] = True
        ranked = sorted(np.nonzero(kept[n])[0].tolist(), key=lambda k: (-conf[n, k], k))
        dead = [k for k in range(K) if not kept[n, k]]
        for i, k in enumerate(dead):
            src[n, k] = ranked[i % len(ranked)]
    return src, kept


# ------------------------------------------------------------------------------- randomness
MASK32 = 0xFFFFFFFF


def philox4x32_10(ctr, key):
    """Philox-4x32 with 10 rounds (Salmon et al., SC'11), vectorised over uint64 arrays
    holding 32-bit lanes.  ctr: 4 arrays, key: 2 ints.  The same published bijection the
    product kernels use for their counter-based fire masks."""
    M0, M1, W0, W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
    x, y, z, w = (np.asarray(c, dtype=np.uint64) & MASK32 for c in ctr)
    k0, k1 = np.uint64(key[0] & MASK32), np.uint64(key[1] & MASK32)
    for _ in range(10):
        p0 = np.uint64(M0) * x
        p1 = np.uint64(M1) * z
        hi0, lo0 = p0 >> np.uint64(32), p0 & np.uint64(MASK32)
        hi1, lo1 = p1 >> np.uint64(32), p1 & np.uint64(MASK32)
        x, y, z, w = (hi1 ^ y ^ k0) & np.uint64(MASK32), lo1, (hi0 ^ w ^ k1) & np.uint64(MASK32), lo0
        k0 = (k0 + np.uint64(W0)) & np.uint64(MASK32)
        k1 = (k1 + np.uint64(W1)) & np.uint64(MASK32)
    return x, y, z, w


def philox_uniform(seed: int, inst: np.ndarray, cell: np.ndarray, step: int) -> np.ndarray:
    """u in [0, 1) (24 bits) for counter (cell, inst_lo, inst_hi, step), key = seed."""
    inst = np.asarray(inst, dtype=np.int64)
    cell = np.asarray(cell, dtype=np.int64)
    inst, cell = np.broadcast_arrays(inst, cell)
    ctr = (cell.astype(np.uint64), inst.astype(np.uint64) & np.uint64(MASK32),
           (inst.astype(np.uint64) >> np.uint64(32)), np.full(inst.shape, step & MASK32, np.uint64))
    o = philox4x32_10(ctr, (seed & MASK32, (seed >> 32) & MASK32))
    return ((o[0] >> np.uint64(8)).astype(np.float64) * (1.0 / 16777216.0)).astype(F32)


def philox_tagged(seed: int, tag: int, inst: np.ndarray, a: np.ndarray, step: int):
    """The kernel's noise streams: counter (a, inst_lo, inst_hi | tag << 24, step), key seed.
    Returns the four output words."""
    inst = np.asarray(inst, dtype=np.int64)
    a = np.asarray(a, dtype=np.int64)
    inst, a = np.broadcast_arrays(inst, a)
    hi = ((inst.astype(np.uint64) >> np.uint64(32)) & np.uint64(0xFFFFFF)) | np.uint64(tag << 24)
    ctr = (a.astype(np.uint64) & np.uint64(MASK32), inst.astype(np.uint64) & np.uint64(MASK32), hi,
           np.full(inst.shape, step & MASK32, np.uint64))
    return philox4x32_10(ctr, (seed & MASK32, (seed >> 32) & MASK32))


def philox_noise(seed: int, inst_ids: np.ndarray, hw: int, channels: int, step: int, p_t: float,
                 p_s: float, sigma: float) -> np.ndarray:
    """Test-time noise of one step (src/nca/perturb.py:23-40) from the kernel's Philox streams:
    instance hit when u(tag 1) < p_t, cell hit when u(tag 2) < p_s, Gaussian values by Box-Muller
    on the words of tag 3 (counter a = cell * C/4 + channel/4, four channels per draw).
    Returns (B, hw, C) float32."""
    ids = np.asarray(inst_ids, dtype=np.int64)
    B = len(ids)
    u = lambda w: (w >> np.uint64(8)).astype(np.float64) / 16777216.0  # noqa: E731
    act = u(philox_tagged(seed, 1, ids, np.zeros(B, np.int64), step)[0]) < np.float32(p_t)
    cell = u(philox_tagged(seed, 2, ids[:, None], np.arange(hw)[None, :], step)[0]) < np.float32(p_s)
    hit = act[:, None] & cell
    C4 = channels // 4
    a = np.arange(hw)[None, :, None] * C4 + np.arange(C4)[None, None, :]
    o = philox_tagged(seed, 3, ids[:, None, None], a, step)
    u0 = ((o[0] >> np.uint64(8)).astype(np.float64) + 0.5) / 16777216.0
    v0 = (o[1] >> np.uint64(8)).astype(np.float64) / 16777216.0
    u1 = ((o[2] >> np.uint64(8)).astype(np.float64) + 0.5) / 16777216.0
    v1 = (o[3] >> np.uint64(8)).astype(np.float64) / 16777216.0
    r0, r1 = np.sqrt(-2.0 * np.log(u0)), np.sqrt(-2.0 * np.log(u1))
    z = np.stack([r0 * np.cos(2 * np.pi * v0), r0 * np.sin(2 * np.pi * v0),
                  r1 * np.cos(2 * np.pi * v1), r1 * np.sin(2 * np.pi * v1)], axis=-1)
    z = (z.reshape(B, hw, channels) * sigma).astype(F32)
    return np.where(hit[:, :, None], z, F32(0))


def philox_masks(seed: int, inst_offset: int, n_inst: int, hw: int, step: int, p: float):
    inst = inst_offset + np.arange(n_inst)[:, None]
    cell = np.arange(hw)[None, :]
    return philox_uniform(seed, inst, cell, step) < F32(p)


def adaptive_prob(conf, scale=0.9, bias=0.1):
    """The benchmark's continuous adaptive rule p = scale * (1 - conf) + bias, applied to the
    reference's per-cell confidence (src/nca/model.py:624-629) instead of the reference's
    threshold rule (src/nca/model.py:587-593)."""
    return (F32(scale) * (F32(1) - conf) + F32(bias)).astype(F32)


# ---------------------------------------------------------------------------------- rollout
def rollout(p: dict, inputs, given, k: int, depth: int, *, channels: int, masks=None, seed=0,
            p_fire=0.5, fire="external", inst_offset=0, uniforms=None, adaptive=None,
            prune_every=0, n_cap=2, targets=None, threshold=None, noise=None, damage=None):
    """Rollout of the benchmark configs (src/nca/rollout.py:86-305 restricted to one pass, no
    noise/damage): boards repeated k times, `depth` steps, then decoded boards and board
    confidences.  fire: 'external' (masks (depth, B, H, W) {0,1}), 'philox' (kernel stream),
    'adaptive_uniform' (uniforms (depth, B, H, W)), 'adaptive_philox'.  prune_every > 0 applies
    niche_cap_refill every prune_every steps.  threshold = (p_low, tau, given_confident) selects
    the reference's threshold rule (src/nca/model.py:566-593) for the adaptive fire modes;
    noise = dict(p_t, p_s, sigma, until) adds philox_noise on steps < until; damage = (t, masks
    (n_boards, H, W) bool) zeroes the masked cells before step t and re-clamps
    (src/nca/rollout.py:206-212)."""
    inputs_k = np.repeat(inputs, k, axis=0)
    given_k = np.repeat(given, k, axis=0)
    x, g4, clamp = init_state(inputs_k, given_k, p, channels)
    B, _, H, W = x.shape
    xs = np.ascontiguousarray(x.transpose(0, 2, 3, 1))
    clamp_s = np.ascontiguousarray(clamp.transpose(0, 2, 3, 1))
    nchw = lambda a: np.ascontiguousarray(a.transpose(0, 3, 1, 2))  # noqa: E731
    updates = np.zeros(B, dtype=np.int64)
    for t in range(depth):
        if damage is not None and t == damage[0]:
            dm = np.repeat(np.asarray(damage[1], bool), k, axis=0)
            xs[dm] = 0.0
            sl = slice(p["in_off"], p["in_off"] + clamp_s.shape[-1])
            xs[..., sl] = np.where(given_k[..., None], clamp_s, xs[..., sl])
        if fire == "external":
            fm = masks[t].reshape(B, H, W) != 0
        elif fire == "philox":
            fm = philox_masks(seed, inst_offset, B, H * W, t, p_fire).reshape(B, H, W)
        else:
            if fire == "adaptive_uniform":
                u = uniforms[t].reshape(B, H, W)
            else:
                u = philox_uniform(seed, inst_offset + np.arange(B)[:, None], np.arange(H * W)[None, :],
                                   t).reshape(B, H, W)
            conf = confidence(nchw(xs), p)
            if threshold is not None:
                p_low, tau, given_conf = threshold
                confident = conf > F32(tau)
                if given_conf:
                    confident = confident | given_k
                fm = u < np.where(confident, F32(p_low), F32(p_fire))
            else:
                a = adaptive or (0.9, 0.1)
                fm = u < adaptive_prob(conf, *a)
        updates += fm.reshape(B, -1).sum(axis=1)
        nz = None
        if noise is not None and t < noise["until"]:
            nz = philox_noise(seed, inst_offset + np.arange(B), H * W, xs.shape[-1], t, noise["p_t"],
                              noise["p_s"], noise["sigma"]).reshape(B, H, W, -1)
        xs = step_nhwc(xs, given_k, clamp_s, fm, p, nz)
        if prune_every and (t + 1) % prune_every == 0 and (t + 1) < depth:
            x = nchw(xs)
            dec = decode_boards(x, given_k, inputs_k, p).reshape(-1, k, H * W)
            conf = board_confidence(x, p).reshape(-1, k)
            src, _ = niche_cap_refill(dec, conf, n_cap)
            flat = (src + np.arange(src.shape[0])[:, None] * k).reshape(-1)
            xs = xs[flat].copy()
            updates = updates[flat].copy()
    x = nchw(xs)
    dec = decode_boards(x, given_k, inputs_k, p)
    return {"x": x, "decoded": dec, "conf": board_confidence(x, p), "updates": updates}


def rollout_halving(p: dict, inputs, given, k: int, depth: int, *, channels: int, seed=0,
                    p_fire=0.5, m=4, n_cap=3, inst_offset=0):
    """Rollout with the reference's pruning (src/nca/rollout.py:154-158, 249-275): at the m - 1
    checkpoints i * (depth // m) the alive trials of every board are halved by
    niche_capped_pruning with rng = default_rng(seed) (rollout.py:103) and the batch is compacted.
    Firing is the kernel's Philox stream keyed by the trial's original index, so a compacted
    trial keeps its stream.  Returns decoded (B, H, W), conf (B,), updates (B,), alive (B,) by
    original index; a pruned trial keeps its values from the checkpoint where it left."""
    rng = np.random.default_rng(seed)
    inputs_k = np.repeat(inputs, k, axis=0)
    given_k = np.repeat(given, k, axis=0)
    x, _, clamp = init_state(inputs_k, given_k, p, channels)
    B, _, H, W = x.shape
    n = B // k
    xs = np.ascontiguousarray(x.transpose(0, 2, 3, 1))
    clamp_s = np.ascontiguousarray(clamp.transpose(0, 2, 3, 1))
    nchw = lambda a: np.ascontiguousarray(a.transpose(0, 3, 1, 2))  # noqa: E731
    dt = depth // m
    checkpoints = {i * dt for i in range(1, m)}
    idx = np.arange(B)
    updates = np.zeros(B, dtype=np.int64)
    out_dec = np.zeros((B, H, W), dtype=np.int64)
    out_conf = np.zeros(B, dtype=F32)
    out_upd = np.zeros(B, dtype=np.int64)
    alive = np.ones(B, dtype=bool)
    for t in range(depth):
        fm = philox_uniform(seed, inst_offset + idx[:, None], np.arange(H * W)[None, :], t)
        fm = (fm < F32(p_fire)).reshape(-1, H, W)
        updates += fm.reshape(len(idx), -1).sum(axis=1)
        xs = step_nhwc(xs, given_k[idx], clamp_s[idx], fm, p)
        if (t + 1) in checkpoints:
            x = nchw(xs)
            dec = decode_boards(x, given_k[idx], inputs_k[idx], p)
            conf = board_confidence(x, p)
            dec_full = np.zeros((B, H, W), dtype=np.int64)
            conf_full = np.full(B, -np.inf, dtype=F32)
            alive_full = np.zeros(B, dtype=bool)
            dec_full[idx], conf_full[idx], alive_full[idx] = dec, conf, True
            keep_full = niche_capped_pruning(dec_full.reshape(n, k, H, W), conf_full.reshape(n, k),
                                             alive_full.reshape(n, k), n_cap, rng.permutation)
            keep = keep_full.reshape(B)[idx]
            drop = ~keep
            out_dec[idx[drop]] = dec[drop]
            out_conf[idx[drop]] = conf[drop]
            out_upd[idx[drop]] = updates[drop]
            alive[idx[drop]] = False
            xs, updates, idx = xs[keep].copy(), updates[keep].copy(), idx[keep]
    x = nchw(xs)
    out_dec[idx] = decode_boards(x, given_k[idx], inputs_k[idx], p)
    out_conf[idx] = board_confidence(x, p)
    out_upd[idx] = updates
    return {"decoded": out_dec, "conf": out_conf, "updates": out_upd, "alive": alive}


def params_from_arrays(d: dict, cfg) -> dict:
    """Oracle parameter dict from the reference-named arrays of a model config (a state dict of
    the reference's NCA: perceive.weight, update.fc1/fc2, and head.* or out_embed, pad_vec)."""
    n_out = len(cfg.output_tokens)
    p = {
        "taps": np.asarray(d["perceive.weight"], F32).reshape(-1, 9),
        "w1": np.asarray(d["update.fc1.weight"], F32).reshape(d["update.fc1.weight"].shape[0], -1),
        "b1": np.asarray(d["update.fc1.bias"], F32),
        "w2": np.asarray(d["update.fc2.weight"], F32).reshape(d["update.fc2.weight"].shape[0], -1),
        "b2": np.asarray(d["update.fc2.bias"], F32),
        "out_tokens": np.asarray(cfg.output_tokens),
        "in_off": cfg.in_offset,
        "out_off": cfg.out_offset,
        "c_out": cfg.c_out,
        "embed": np.asarray(d["embed"], F32) if "embed" in d else np.eye(cfg.vocab_size, cfg.c_in, dtype=F32),
        "head": cfg.head,
    }
    if cfg.head == "l2":
        p["out_embed"] = np.asarray(d["out_embed"], F32).reshape(n_out, -1)
    else:
        p["head_w"] = np.asarray(d["head.weight"], F32).reshape(n_out, -1)
        p["head_b"] = np.asarray(d["head.bias"], F32)
    if getattr(cfg, "padding", "zero") == "wall":
        p["pad"] = np.asarray(d["pad_vec"], F32)
    return p
