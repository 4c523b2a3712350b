"""CPU oracle for the DWA retrieval + assembly hot path of theorionic/matrix.

TEST INFRASTRUCTURE ONLY.  This module restates, in NumPy, the arithmetic of the
reference's JAX code so that the CUDA path can be checked against it.  Only the
tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import it,
and only as the checker / the timed CPU port.  The product path
(``matrix_b200``) never imports or calls anything here.

Every function cites the reference file:line it follows (paths relative to the
reference project root).  Arithmetic is done in the dtype of the inputs (pass
float64 arrays for a high-precision oracle, float32 arrays for the reference's
own precision).

Pinning: the outputs of this restatement are checked against golden vectors
produced by executing the reference's own source files
(``src/dwa/retrieval.py``, ``src/dwa/assembly_pallas.py``) under a NumPy stand-in
for ``jax``/``flax`` (``tests/golden/make_golden.py``), and against the
invariants the reference's tests assert (``tests/test_retrieval.py``,
``tests/test_assembly.py``).  The reference ships no golden vectors of its own
and JAX is not installable here, so XLA itself never ran; see
``tests/golden/make_golden.py`` for what that pin does and does not cover.

Extensions beyond the reference (each reduces exactly to the reference when
switched off):

* ``list_offsets``: CSR list boundaries so lists may have unequal sizes
  (the reference only supports ``N % C == 0`` equal lists, config.py:64-67).
* ``tie_break="index"``: among exactly equal scores, prefer the lower global
  pool index instead of the lower candidate position (``lax.top_k`` position
  order, retrieval.py:144-145).  The two agree whenever no two candidate scores
  are bit-identical.
"""

from __future__ import annotations

import numpy as np

EPS = 1e-8  # retrieval.py:66,86,103,115 and assembly_pallas :152,155 use +1e-8


# ---------------------------------------------------------------------------
# jnp / lax primitives with the reference's semantics
# ---------------------------------------------------------------------------

def l2_normalize(x: np.ndarray) -> np.ndarray:
    """``x / (||x||_2 + 1e-8)`` over the last axis (retrieval.py:66, 85-87, 102-104)."""
    return x / (np.linalg.norm(x, axis=-1, keepdims=True) + x.dtype.type(EPS))


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """``jax.nn.softmax``: ``exp(x - max) / sum(exp(x - max))``."""
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=axis, keepdims=True)


def sigmoid(x: np.ndarray) -> np.ndarray:
    """``jax.nn.sigmoid`` (retrieval.py:150)."""
    return 1.0 / (1.0 + np.exp(-x))


def top_k(x: np.ndarray, k: int, tie_key: np.ndarray | None = None):
    """``jax.lax.top_k`` over the last axis: values descending.

    Ties between bit-identical values go to the lower *position* (XLA's rule),
    or, when ``tie_key`` (same shape as ``x``) is given, to the lower tie key
    (used for the lower-global-index rule).
    Returns ``(values, positions)``.
    """
    if tie_key is None:
        order = np.argsort(-x, axis=-1, kind="stable")
    else:
        # lexsort sorts by the last key first: primary = -x, secondary = tie_key
        order = np.lexsort((tie_key, -x), axis=-1)
    pos = order[..., :k]
    return np.take_along_axis(x, pos, axis=-1), pos


# ---------------------------------------------------------------------------
# Retrieval: MultiAspectRetrieval.__call__ (retrieval.py:48-159)
# ---------------------------------------------------------------------------

def equal_list_offsets(N: int, C: int) -> np.ndarray:
    """List c = rows ``[c*N/C, (c+1)*N/C)`` (retrieval.py:94-98, config.py:64-67)."""
    assert N % C == 0, "equal lists need N % C == 0 (config.py:64-67)"
    return (np.arange(C + 1, dtype=np.int64) * (N // C)).astype(np.int64)


def aspect_queries(W_Q: np.ndarray, z: np.ndarray) -> np.ndarray:
    """Normalised aspect queries ``q̂[b,s,:]`` (retrieval.py:64-66)."""
    queries = np.einsum("ska,ba->bsk", W_Q, z)
    return l2_normalize(queries)


def coarse_scores(q_norm, w, centroids):
    """``c_score[b,c] = Σ_s w_s q̂[b,s]·ĉ[s,c]`` (retrieval.py:85-89)."""
    c_norm = l2_normalize(centroids)
    c_sim = np.einsum("bsk,sck->bsc", q_norm, c_norm)
    return np.einsum("s,bsc->bc", w, c_sim)


def candidate_lists(top_clusters: np.ndarray, list_offsets: np.ndarray):
    """Candidate pool rows in cluster-rank-major order (retrieval.py:94-98).

    With equal lists this is exactly ``top_clusters[:, :, None] * N_per_C +
    arange(N_per_C)``.  With CSR offsets each query's candidate count may differ;
    the result is a list of 1-D int64 arrays, one per query.
    """
    out = []
    for b in range(top_clusters.shape[0]):
        parts = [np.arange(list_offsets[c], list_offsets[c + 1], dtype=np.int64)
                 for c in top_clusters[b]]
        out.append(np.concatenate(parts) if parts else np.zeros(0, np.int64))
    return out


def fine_scores(q_norm, w, pool_keys, cand):
    """``s_i[n] = Σ_s w_s q̂_s·k̂_s[cand[n]]`` for one query (retrieval.py:100-106).

    ``q_norm`` is ``[S, d_k]`` for that query and ``cand`` the 1-D candidate rows.
    """
    keys_refine = pool_keys[:, cand, :]                        # [S, K_ref, d_k]
    k_norm = l2_normalize(keys_refine)
    sim_ref = np.einsum("sk,snk->sn", q_norm, k_norm)
    return np.einsum("s,sn->n", w, sim_ref)


def full_scores(q_norm, w, pool_keys):
    """``s_full[b,n]`` over every pool row (retrieval.py:114-118, 123-125)."""
    p_norm = l2_normalize(pool_keys)
    sim_all = np.einsum("bsk,snk->bsn", q_norm, p_norm, optimize=True)
    return np.einsum("s,bsn->bn", w, sim_all)


def select(s_i, cand, k, T, lambda_val, tau, is_warmup, tie_break="position"):
    """Warmup / gate selection for one query (retrieval.py:143-156).

    Returns ``(alpha [k], global_idx [k])``.  Gate mode ranks ``raw`` exactly as
    the reference does (``raw`` is monotone in ``s_i`` for ``lambda >= 0``).
    """
    tie = cand if tie_break == "index" else None
    if is_warmup:
        scores, pos = top_k(s_i, k, tie)                      # :144
        alpha = softmax(scores / s_i.dtype.type(T))            # :146
    else:
        g = sigmoid(s_i.dtype.type(lambda_val) * (s_i - s_i.dtype.type(tau)))   # :150
        raw = g * np.exp(s_i / s_i.dtype.type(T))              # :151
        raw = raw / (raw.sum() + s_i.dtype.type(EPS))          # :152
        top_raw, pos = top_k(raw, k, tie)                      # :153
        alpha = top_raw / (top_raw.sum() + s_i.dtype.type(EPS))  # :155
    return alpha, cand[pos]                                    # :145,:154


def retrieve(z, W_Q, aspect_weights, tau, centroids, pool_keys, *, k, m, T,
             lambda_val, is_warmup, use_ivf=True, list_offsets=None,
             tie_break="position", want_soft_full=True, return_internals=False):
    """``MultiAspectRetrieval.__call__`` (retrieval.py:48-159), single device.

    Arguments mirror the module's parameters (``W_Q [S,d_k,d_A]``,
    ``aspect_weights [S]``, ``tau``, ``centroids [S,C,d_k]``) and call arguments
    (``z [B,d_A]``, ``pool_keys [S,N,d_k]``, ``lambda_val``, ``is_warmup``).
    Returns ``(alphas [B,k], indices [B,k] int64, soft_full [B,N] or None)``.
    """
    B = z.shape[0]
    S, N, _ = pool_keys.shape
    q_norm = aspect_queries(W_Q, z)                             # :65-66
    w = softmax(aspect_weights, axis=0)                         # :69
    internals = {"q_norm": q_norm, "w": w}
    soft_full = None
    if use_ivf:
        C = centroids.shape[1]
        if list_offsets is None:
            list_offsets = equal_list_offsets(N, C)
        c_score = coarse_scores(q_norm, w, centroids)           # :85-89
        m_eff = min(m, C)                                       # :90
        _, top_clusters = top_k(c_score, m_eff)                 # :91
        cands = candidate_lists(top_clusters, list_offsets)     # :94-98
        s_list = [fine_scores(q_norm[b], w, pool_keys, cands[b]) for b in range(B)]
        internals.update(c_score=c_score, top_clusters=top_clusters,
                         cands=cands, s_i=s_list)
        if want_soft_full:
            soft_full = softmax(full_scores(q_norm, w, pool_keys) / q_norm.dtype.type(T))  # :114-119
    else:
        s_full = full_scores(q_norm, w, pool_keys)              # :123-125
        cands = [np.arange(N, dtype=np.int64) for _ in range(B)]   # :135-137
        s_list = [s_full[b] for b in range(B)]
        internals.update(cands=cands, s_i=s_list)
        if want_soft_full:
            soft_full = softmax(s_full / q_norm.dtype.type(T))  # :138
    alphas = np.zeros((B, k), dtype=q_norm.dtype)
    indices = np.zeros((B, k), dtype=np.int64)
    for b in range(B):
        alphas[b], indices[b] = select(s_list[b], cands[b], k, T, lambda_val, tau,
                                       is_warmup, tie_break)
    if return_internals:
        return alphas, indices, soft_full, internals
    return alphas, indices, soft_full


def _normalize_bwd(x, g_y):
    """VJP of ``x / (||x|| + 1e-8)`` over the last axis (the gradient of
    ``jnp.linalg.norm`` is ``x / ||x||``)."""
    n = np.linalg.norm(x, axis=-1, keepdims=True)
    d = n + x.dtype.type(EPS)
    return g_y / d - x * np.sum(x * g_y, axis=-1, keepdims=True) / (n * d * d)


def retrieve_bwd(z, W_Q, aspect_weights, tau, centroids, pool_keys, *, k, m, T, lambda_val,
                 is_warmup, g_alphas=None, g_soft_full=None, use_ivf=True, list_offsets=None,
                 tie_break="index"):
    """VJP of ``retrieve`` (retrieval.py:64-158): the cotangents of ``alphas``
    and ``soft_full`` back to ``z``, ``W_Q``, ``aspect_weights``, ``tau`` and
    ``pool_keys``, as ``jax.vjp`` of ``MultiAspectRetrieval.__call__`` gives
    them.  ``indices`` are integers and the coarse top-m and the top-k are
    piecewise constant, so no gradient reaches the centroids; ``lambda_val`` is
    a schedule value, not a parameter.

    Every score the selection or soft_full reads is ``s[b, n] = Σ_s w_s
    q̂[b,s]·k̂[s,n]`` (:100-106, :114-118), so the cotangents are first collected
    per (query, pool row) in ``G [B, N]``:

    * warmup (:144-146): ``α = softmax(top/T)`` puts ``α(g_α - Σ α g_α)/T`` on
      the winners' rows;
    * gate (:150-155): ``raw = σ(λ(s-τ)) e^{s/T}``, ``rn = raw/(Σ raw + 1e-8)``,
      ``α = top(rn)/(Σ top + 1e-8)``: every candidate's row gets
      ``g_raw · raw · (λ(1-σ) + 1/T)`` through the sum over all candidates,
      and ``τ`` gets ``-Σ g_raw · raw · λ(1-σ)``;
    * soft_full (:118-119): ``soft (g_soft - Σ g_soft soft) / T`` on every row.

    Then ``A[b,s] = Σ_n G[b,n] k̂[s,n]`` gives ``g_q̂ = w_s A``, ``g_w[s] =
    Σ_b q̂[b,s]·A[b,s]`` and ``g_k̂[s,n] = w_s Σ_b G[b,n] q̂[b,s]``, followed by
    the normalisation, projection (:65) and softmax (:69) backward.

    Returns ``dict(g_z, g_W_Q, g_aspect_weights, g_tau, g_pool_keys, G)``.
    """
    dt = z.dtype.type
    B = z.shape[0]
    S, N, _ = pool_keys.shape
    queries = np.einsum("ska,ba->bsk", W_Q, z)                  # :65
    q_norm = l2_normalize(queries)                               # :66
    w = softmax(aspect_weights, axis=0)                          # :69
    T_ = dt(T)
    if use_ivf:
        C = centroids.shape[1]
        if list_offsets is None:
            list_offsets = equal_list_offsets(N, C)
        _, top_clusters = top_k(coarse_scores(q_norm, w, centroids), min(m, C))
        cands = candidate_lists(top_clusters, list_offsets)
        s_list = [fine_scores(q_norm[b], w, pool_keys, cands[b]) for b in range(B)]
    else:
        s_full = full_scores(q_norm, w, pool_keys)
        cands = [np.arange(N, dtype=np.int64) for _ in range(B)]
        s_list = [s_full[b] for b in range(B)]
    G = np.zeros((B, N), dtype=z.dtype)
    g_tau = dt(0)
    if g_alphas is not None:
        lam, tau_ = dt(lambda_val), dt(tau)
        for b in range(B):
            s, cand = s_list[b], cands[b]
            tie = cand if tie_break == "index" else None
            if is_warmup:
                top, pos = top_k(s, k, tie)
                alpha = softmax(top / T_)
                ga = g_alphas[b, :len(pos)]
                G[b, cand[pos]] += alpha * (ga - np.sum(alpha * ga)) / T_
            else:
                sg = sigmoid(lam * (s - tau_))
                raw = sg * np.exp(s / T_)
                Zr = raw.sum() + dt(EPS)
                rn = raw / Zr
                top_raw, pos = top_k(rn, k, tie)
                St = top_raw.sum() + dt(EPS)
                ga = g_alphas[b, :len(pos)]
                g_t = ga / St - np.sum(ga * top_raw) / (St * St)
                g_rn = np.zeros_like(s)
                g_rn[pos] = g_t
                g_raw = g_rn / Zr - np.sum(g_rn * raw) / (Zr * Zr)
                G[b, cand] += g_raw * raw * (lam * (1 - sg) + 1 / T_)
                g_tau += np.sum(g_raw * raw * (-lam * (1 - sg)))
    if g_soft_full is not None:
        soft = softmax(full_scores(q_norm, w, pool_keys) / T_)
        G += soft * (g_soft_full - np.sum(g_soft_full * soft, axis=-1, keepdims=True)) / T_
    k_norm = l2_normalize(pool_keys)
    A = np.einsum("bn,snk->bsk", G, k_norm)
    g_qn = w[None, :, None] * A
    g_w = np.einsum("bsk,bsk->s", q_norm, A)
    g_kn = np.einsum("bn,s,bsk->snk", G, w, q_norm)
    g_queries = _normalize_bwd(queries, g_qn)
    return dict(
        g_z=np.einsum("bsk,ska->ba", g_queries, W_Q),
        g_W_Q=np.einsum("bsk,ba->ska", g_queries, z),
        g_aspect_weights=w * (g_w - np.sum(w * g_w)),
        g_tau=g_tau,
        g_pool_keys=_normalize_bwd(pool_keys, g_kn),
        G=G,
    )


# ---------------------------------------------------------------------------
# Auxiliary losses: aux_losses (losses.py:9-73) and their VJP
# ---------------------------------------------------------------------------

def aux_losses(alphas, indices, pool_keys, W, W_base, soft_full, *, lambda_util, lambda_div,
               lambda_norm, lambda_sparse):
    """``aux_losses`` (losses.py:9-73), literally: ``l_util = N Σ f P``
    (:35-38), ``l_div`` the mean upper-triangle cosine of the aspect-mean
    retrieved keys (:42-50), ``l_norm = mean_b ||W_b - W_base||²`` (:53-54),
    ``l_sparse`` the mean entropy of the clipped alphas (:57-58) and the
    weighted total (:66-71)."""
    B, k = alphas.shape
    N = soft_full.shape[-1]
    dt = alphas.dtype.type
    f = np.zeros(N, dtype=alphas.dtype)
    np.add.at(f, indices.reshape(-1), dt(1))
    f = f / dt(B * k)
    P = soft_full.mean(axis=0)
    l_util = dt(N) * np.dot(f, P)
    rk = pool_keys[:, indices, :].transpose(1, 2, 0, 3).mean(axis=2)        # [B, k, d_k]
    rkn = l2_normalize(rk)
    cos = np.einsum("bkd,bld->bkl", rkn, rkn)
    mask = np.triu(np.ones((k, k), dtype=bool), k=1)
    l_div = (cos * mask[None]).sum() / (mask.sum() * B + dt(EPS))
    l_norm = ((W - W_base[None]) ** 2).sum(axis=(-1, -2)).mean()
    a = np.clip(alphas, dt(1e-8), dt(1.0))
    l_sparse = -(a * np.log(a)).sum(axis=-1).mean()
    total = (dt(lambda_util) * l_util + dt(lambda_div) * l_div + dt(lambda_norm) * l_norm
             + dt(lambda_sparse) * l_sparse)
    return dict(l_util=l_util, l_div=l_div, l_norm=l_norm, l_sparse=l_sparse, total_aux=total)


def aux_losses_bwd(alphas, indices, pool_keys, W, W_base, soft_full, *, lambda_util, lambda_div,
                   lambda_norm, lambda_sparse):
    """Gradients of ``total_aux`` (losses.py:66-71) w.r.t. alphas, soft_full, W,
    W_base and pool_keys, as ``jax.grad`` gives them:

    * ``g_soft[b, n] = λ_util N f_n / B`` (:38);
    * ``l_div``: ``g_r̂_i = c (U - r̂_i)`` with ``U = Σ_j r̂_j`` and
      ``c = λ_div / (B k(k-1)/2 + 1e-8)``, then the normalisation VJP and
      ``1/S`` into every aspect's row ``indices[b, i]`` (duplicates add);
    * ``g_W = 2 λ_norm (W - W_base) / B``, ``g_W_base = -Σ_b g_W``;
    * ``g_α = -λ_sparse (log a + 1) / B`` times the gradient of
      ``jnp.clip`` (1 inside (1e-8, 1), 1/2 on a bound, 0 outside).
    """
    B, k = alphas.shape
    S, N, d_k = pool_keys.shape
    dt = alphas.dtype.type
    f = np.zeros(N, dtype=alphas.dtype)
    np.add.at(f, indices.reshape(-1), dt(1))
    f = f / dt(B * k)
    g_soft = np.broadcast_to(dt(lambda_util) * dt(N) * f / dt(B), (B, N)).copy()
    rk = pool_keys[:, indices, :].transpose(1, 2, 0, 3).mean(axis=2)        # [B, k, d_k]
    rkn = l2_normalize(rk)
    c = dt(lambda_div) / (dt(k * (k - 1) // 2 * B) + dt(EPS))
    g_rkn = c * (rkn.sum(axis=1, keepdims=True) - rkn)
    g_rk = _normalize_bwd(rk, g_rkn)
    g_keys = np.zeros_like(pool_keys)
    for s in range(S):
        np.add.at(g_keys[s], indices.reshape(-1), g_rk.reshape(-1, d_k) / dt(S))
    g_W = dt(2 * lambda_norm / B) * (W - W_base[None])
    lo, hi = dt(1e-8), dt(1.0)
    a = np.clip(alphas, lo, hi)
    clip_grad = np.where((alphas > lo) & (alphas < hi), dt(1), np.where((alphas == lo) | (alphas == hi), dt(0.5), dt(0)))
    g_alphas = -dt(lambda_sparse) * (np.log(a) + 1) / dt(B) * clip_grad
    return dict(g_alphas=g_alphas, g_soft_full=g_soft, g_W=g_W, g_W_base=-g_W.sum(axis=0),
                g_pool_keys=g_keys)


# ---------------------------------------------------------------------------
# Row-sharded retrieval: one rank's summary and the merge (extension; with one
# rank it reduces to ``retrieve`` with tie_break="index")
# ---------------------------------------------------------------------------

def summary_width(k: int) -> int:
    return 2 * k + 3


def retrieve_local(z, W_Q, aspect_weights, tau, centroids, local_keys, *, row_lo, k, m, T,
                   lambda_val, is_warmup, use_ivf=True, list_offsets=None, n_global=None,
                   want_soft_full=True):
    """One rank's part of a row-sharded call: the rank holds the keys of pool rows
    ``[row_lo, row_lo + N_local)``; the top-m lists are chosen exactly as in
    ``retrieve`` (retrieval.py:85-98) and only their rows held here are scored
    (:100-106).  Returns ``(summary [B, 2k+3], s_full_local [B, N_local] or None)``:
    the rank's top-k (scores best first, global rows as floats), the partial sum of
    the unnormalised gate ``raw`` (:150-151), and the max / sum of exp of s/T over
    its rows (:114-119)."""
    B = z.shape[0]
    S, n_loc, _ = local_keys.shape
    f = local_keys.dtype.type
    q_norm = aspect_queries(W_Q, z)
    w = softmax(aspect_weights, axis=0)
    row_hi = row_lo + n_loc
    if use_ivf:
        C = centroids.shape[1]
        if list_offsets is None:
            list_offsets = equal_list_offsets(n_global, C)
        _, top_clusters = top_k(coarse_scores(q_norm, w, centroids), min(m, C))
        cands = [c[(c >= row_lo) & (c < row_hi)] for c in candidate_lists(top_clusters, list_offsets)]
    else:
        cands = [np.arange(row_lo, row_hi, dtype=np.int64) for _ in range(B)]
    W = summary_width(k)
    summary = np.zeros((B, W), dtype=np.float64)
    for b in range(B):
        c = cands[b]
        s = fine_scores(q_norm[b], w, local_keys, c - row_lo) if c.size else np.zeros(0, f)
        if is_warmup:
            rank, zpart = s, 0.0
        else:
            raw = sigmoid(f(lambda_val) * (s - f(tau))) * np.exp(s / f(T))
            rank, zpart = raw, float(raw.sum())
        _, pos = top_k(rank, min(k, c.size), c)
        got = pos.size
        summary[b, :k] = -np.inf
        summary[b, k:2 * k] = -1
        summary[b, :got] = s[pos]
        summary[b, k:k + got] = c[pos]
        summary[b, 2 * k] = zpart
    s_loc = None
    if want_soft_full:
        s_loc = full_scores(q_norm, w, local_keys)
        x = s_loc / f(T)
        mx = x.max(axis=1) if n_loc else np.full(B, -np.inf)
        summary[:, 2 * k + 1] = mx
        summary[:, 2 * k + 2] = np.exp(x - mx[:, None]).sum(axis=1) if n_loc else 0.0
    else:
        summary[:, 2 * k + 1] = -np.inf
        summary[:, 2 * k + 2] = 0.0
    return summary, s_loc


def merge_summaries(summaries, *, k, T, lambda_val, tau, is_warmup):
    """Merge of the ranks' summaries ``[P, B, 2k+3]``: the global top-k (ties to the
    lower pool row), alphas by retrieval.py:146 (warmup) or :152-155 (gate, with
    the gate sum added over ranks), and the combined soft_full statistics.
    Returns ``(alphas [B,k], indices [B,k], stats [B,2] = (max, sum exp))``."""
    P, B, _ = summaries.shape
    alphas = np.zeros((B, k))
    indices = np.zeros((B, k), dtype=np.int64)
    stats = np.zeros((B, 2))
    for b in range(B):
        s = summaries[:, b, :k].reshape(-1)
        rows = summaries[:, b, k:2 * k].reshape(-1).astype(np.int64)
        ok = rows >= 0
        s, rows = s[ok], rows[ok]
        Z = summaries[:, b, 2 * k].sum()
        if is_warmup:
            top, pos = top_k(s, k, rows)
            alphas[b] = softmax(top / T)
        else:
            raw = sigmoid(lambda_val * (s - tau)) * np.exp(s / T) / (Z + EPS)
            top_raw, pos = top_k(raw, k, rows)
            alphas[b] = top_raw / (top_raw.sum() + EPS)
        indices[b] = rows[pos]
        mx = summaries[:, b, 2 * k + 1]
        M = mx.max()
        stats[b] = M, (summaries[:, b, 2 * k + 2] * np.exp(np.where(np.isfinite(mx), mx - M, -np.inf))).sum()
    return alphas, indices, stats


# ---------------------------------------------------------------------------
# Gather (model.py:184-195) and key cache (assembly_pallas.py:392-400)
# ---------------------------------------------------------------------------

def gather(pool_vectors, indices, out_dtype=np.float32):
    """``pool_vecs[indices]`` then the cast to float32 (model.py:193-195)."""
    return pool_vectors[indices].astype(out_dtype)


def compute_key_cache(pool_vectors, key_proj):
    """``einsum("nd,sda->sna")`` (assembly_pallas.py:392-400, pool.py:37-44)."""
    return np.einsum("nd,sda->sna", pool_vectors, key_proj)


def centroid_ema(centroids, keys, list_offsets, decay=0.9):
    """Centroid update of train.py:318-328: ``decay * c + (1 - decay) * mean`` of
    each list's keys (the reference reshapes equal lists ``[S, C, N/C, d_k]`` and
    takes the mean over axis 2; CSR lists are the extension).  Empty lists keep
    their centroid."""
    out = centroids.copy()
    for c in range(centroids.shape[1]):
        lo, hi = int(list_offsets[c]), int(list_offsets[c + 1])
        if hi > lo:
            out[:, c] = decay * centroids[:, c] + (1 - decay) * keys[:, lo:hi].mean(axis=1)
    return out


# ---------------------------------------------------------------------------
# RMSNorm after the assembly (assembly.py:29, model.py:207-219)
# ---------------------------------------------------------------------------
# The reference calls flax's ``nnx.RMSNorm(d_B)``; flax is not vendored and its
# version is not pinned (pyproject.toml:7 lists no dependencies).  Restated from
# flax's published algorithm: statistics ``mean(x^2)`` over the feature axis in
# at least float32, ``mul = rsqrt(var + epsilon) * scale`` (epsilon = 1e-6 by
# default, scale initialised to ones), ``y = x * mul``.

def rms_norm(x, scale, eps=1e-6):
    var = np.mean(np.square(x), axis=-1, keepdims=True)
    return x * (1.0 / np.sqrt(var + eps) * scale)


def rms_norm_bwd(x, scale, g, eps=1e-6):
    """VJP of ``rms_norm`` w.r.t. ``x`` and ``scale`` (``g`` = dL/dy)."""
    d = x.shape[-1]
    r = 1.0 / np.sqrt(np.mean(np.square(x), axis=-1, keepdims=True) + eps)
    dot = np.sum(g * scale * x, axis=-1, keepdims=True)
    g_x = r * scale * g - (r ** 3 / d) * x * dot
    g_scale = np.sum((g * x * r).reshape(-1, d), axis=0)
    return g_x, g_scale


# ---------------------------------------------------------------------------
# Assembly forward: assemble_jax (assembly_pallas.py:42-75)
# ---------------------------------------------------------------------------

def factor_split(d_B: int, r: int, d_A: int):
    """``(s1, s2, s3)`` (config.py:159-165)."""
    s1 = d_B * r
    s2 = s1 + r * d_A
    return s1, s2, s2 + d_B


def split_factors(gathered, d_B, r, d_A):
    """U ``[B,k,d_B,r]``, V ``[B,k,r,d_A]``, b ``[B,k,d_B]`` (assembly_pallas.py:54-60)."""
    B, k, _ = gathered.shape
    s1, s2, s3 = factor_split(d_B, r, d_A)
    U = gathered[:, :, :s1].reshape(B, k, d_B, r)
    V = gathered[:, :, s1:s2].reshape(B, k, r, d_A)
    b_vec = gathered[:, :, s2:s3]
    return U, V, b_vec


def assemble(gathered, alphas, h_A, W_base, b_base, gamma, d_B, r, d_A):
    """``assemble_jax`` (assembly_pallas.py:42-75).  Returns ``(h_mid, W)``."""
    B, k, _ = gathered.shape
    U, V, b_vec = split_factors(gathered, d_B, r, d_A)
    aU = alphas[:, :, None, None] * U                                   # :63
    delta_W = np.matmul(aU.reshape(B * k, d_B, r),
                        V.reshape(B * k, r, d_A)).reshape(B, k, d_B, d_A).sum(1)  # :64-66
    W = W_base[None, ...] + delta_W                                     # :67
    delta_b = (alphas[:, :, None] * b_vec).sum(1)                       # :69
    bias = b_base[None, :] + delta_b                                    # :70
    h_res = np.matmul(h_A, W.transpose(0, 2, 1))                        # :73
    h_mid = h_A + gamma * h_res + bias[:, None, :]                      # :74
    return h_mid, W


# ---------------------------------------------------------------------------
# Assembly backward: _pallas_assemble_bwd (assembly_pallas.py:246-329)
# ---------------------------------------------------------------------------

def assemble_bwd(gathered, alphas, h_A, W, gamma, g_hmid, g_W_out, d_B, r, d_A,
                 batch_chunk: int | None = None):
    """Analytic VJP of the assembly (assembly_pallas.py:246-329).

    Returns ``(g_gathered [B,k,D], g_alpha [B,k], g_hA [B,T,d_A],
    g_W_base [d_B,d_A], g_b_base [d_B], g_gamma ())``.  ``g_W_out`` may be
    ``None`` for a zero cotangent of the ``W`` output.  ``batch_chunk`` only
    bounds the memory of the ``UV [B,k,d_B,d_A]`` temporary (:293-298); the
    arithmetic per element is unchanged.
    """
    B, k, D = gathered.shape
    s1, s2, s3 = factor_split(d_B, r, d_A)
    if g_W_out is None:
        g_W_out = np.zeros_like(W)
    U, V, b_vec = split_factors(gathered, d_B, r, d_A)                 # :267-269
    h_res = np.matmul(h_A, W.transpose(0, 2, 1))                       # :272
    g_gamma = np.sum(g_hmid * h_res)                                   # :275
    g_bias = g_hmid.sum(axis=1)                                        # :276
    g_h_res = gamma * g_hmid                                           # :277
    g_W_hres = np.einsum("btj,bti->bji", g_h_res, h_A, optimize=True)  # :281
    g_hA_hres = np.einsum("btj,bji->bti", g_h_res, W, optimize=True)   # :283
    g_hA = g_hmid + g_hA_hres                                          # :285
    g_W_total = g_W_hres + g_W_out                                     # :288
    g_W_base = g_W_total.sum(0)                                        # :289
    g_delta_W = g_W_total                                              # :290
    step = batch_chunk or B
    g_alpha_dW = np.zeros((B, k), dtype=g_delta_W.dtype)
    for b0 in range(0, B, step):
        b1 = min(B, b0 + step)
        nb = b1 - b0
        UV = np.matmul(U[b0:b1].reshape(nb * k, d_B, r),
                       V[b0:b1].reshape(nb * k, r, d_A)).reshape(nb, k, d_B, d_A)  # :293-295
        g_alpha_dW[b0:b1] = np.einsum("bkji,bji->bk", UV, g_delta_W[b0:b1], optimize=True)  # :298
    g_U = alphas[:, :, None, None] * np.matmul(g_delta_W[:, None, :, :],
                                               V.transpose(0, 1, 3, 2))          # :303-305
    g_V = alphas[:, :, None, None] * np.matmul(U.transpose(0, 1, 3, 2),
                                               g_delta_W[:, None, :, :])         # :310-312
    g_b_base = g_bias.sum(0)                                           # :315
    g_alpha_bias = (b_vec * g_bias[:, None, :]).sum(-1)                # :316
    g_b_vec = alphas[:, :, None] * g_bias[:, None, :]                  # :317
    g_alpha = g_alpha_dW + g_alpha_bias                                # :319
    g_gathered = np.concatenate([                                      # :322-327
        g_U.reshape(B, k, s1),
        g_V.reshape(B, k, s2 - s1),
        g_b_vec,
        np.zeros((B, k, D - s3), dtype=gathered.dtype),
    ], axis=-1)
    return g_gathered, g_alpha, g_hA, g_W_base, g_b_base, g_gamma


def pallas_forward(gathered, alphas, h_A, W_base, b_base, gamma, d_B, r, d_A):
    """The Pallas kernel's arithmetic (assembly_pallas.py:85-181), in the
    pre-factored order it uses: ``hA + γ(hA·W_baseᵀ + (hA·V_sᵀ)·U_f) + pb``.

    Equal to :func:`assemble` up to rounding for every B (the reference's Pallas
    grid leaves rows ``B - B % 8 .. B`` unwritten when ``B > 8`` and
    ``B % 8 != 0``, :100,131; this restatement computes them).
    """
    B, k, _ = gathered.shape
    kr = k * r
    U, V, b_vec = split_factors(gathered, d_B, r, d_A)
    V_scaled = (alphas[:, :, None, None] * V).reshape(B, kr, d_A)     # :168
    U_flat = U.transpose(0, 1, 3, 2).reshape(B, kr, d_B)              # :169
    pb = b_base + np.einsum("bk,bkd->bd", alphas, b_vec)              # :170-171
    h_V = np.matmul(h_A, V_scaled.transpose(0, 2, 1))                  # :113
    h_res_delta = np.matmul(h_V, U_flat)                               # :114
    h_base = np.matmul(h_A, W_base.T)                                  # :115
    return h_A + gamma * (h_base + h_res_delta) + pb[:, None, :]       # :117
