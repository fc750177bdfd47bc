"""Float64 kernel evaluation from the gpb200 int32 kernel program.

Restates the per-pair expressions the reference codegen emits
(mojogp/codegen_engine/expressions.py:77-420) after its numerical-stability
pass (codegen_engine/passes/numerical_stability.py:13-112):
  * exp(max(arg, -20)) clamp on Matern-1/2 ARD, Matern-3/2, Matern-5/2;
  * r = sqrt(max(s + 1e-20, 1e-20)) for the Matern family;
  * Periodic: os * exp(-2 * sum_k sin^2(pi diff_k / p) / l_k) (l, not l^2);
  * Polynomial: os * (dot + offset)^degree with a fixed integer degree.
Composition (sum / product / scale) follows kernel.py:756-802.
"""
from __future__ import annotations

import numpy as np

LEAF, SUM, PROD, SCALE = 1, 2, 3, 4
RBF, M12, M32, M52, RQ, PER, LIN, POLY = range(8)


def leaf_num_params(kt: int, ard: bool, nd: int) -> int:
    if kt in (RBF, M12, M32, M52, LIN):
        return (nd if ard else 1) + 1
    if kt in (RQ, PER):
        return (nd if ard else 1) + 2
    if kt == POLY:
        return nd + 3 if ard else 3
    raise ValueError(kt)


def parse(spec):
    """Decode the post-order program into a list of node tuples."""
    spec = [int(x) for x in spec]
    assert spec[0] == 1, "spec version"
    P, nn = spec[1], spec[2]
    pos, nodes = 3, []
    for _ in range(nn):
        op = spec[pos]
        pos += 1
        if op == LEAF:
            kt, ard, pofs, nd = spec[pos:pos + 4]
            pos += 4
            dims = spec[pos:pos + nd]
            pos += nd
            nodes.append(("leaf", kt, bool(ard), pofs, dims))
        elif op == SCALE:
            nodes.append(("scale", spec[pos]))
            pos += 1
        elif op == SUM:
            nodes.append(("sum",))
        elif op == PROD:
            nodes.append(("prod",))
        else:
            raise ValueError(op)
    assert pos == len(spec)
    return P, nodes


def _leaf(kt, ard, p, X1, X2, want_grad):
    """Returns K [n1, n2] and (if want_grad) list of dK/dtheta for leaf params."""
    nd = X1.shape[1]
    grads = []
    if kt in (RBF, M12, M32, M52, RQ):
        nl = nd if ard else 1
        ell = p[:nd] if ard else np.full(nd, p[0])
        if want_grad:
            diff = X1[:, None, :] - X2[None, :, :]  # [n1, n2, nd]
            dl = diff / ell
            sq = dl * dl
            s = sq.sum(axis=2)
        else:
            # Same sum, one input dim at a time: [n1, n2] memory instead of
            # [n1, n2, nd], so row samples against 1e6 columns fit.
            a1, a2 = X1 / ell, np.ascontiguousarray((X2 / ell).T)
            s = np.zeros((X1.shape[0], X2.shape[0]))
            dk = np.empty_like(s)
            for k in range(nd):
                np.subtract(a1[:, k, None], a2[k][None, :], out=dk)
                np.multiply(dk, dk, out=dk)
                s += dk
        if kt == RQ:
            alpha, os = p[nl], p[nl + 1]
            z = s / (2.0 * alpha)
            base = 1.0 + z
            kap = base ** (-alpha)
            psi = kap / base
            K = os * kap
            g_alpha = K * (z / base - np.log(base))
            os_idx = nl + 1
        else:
            os = p[nl]
            os_idx = nl
            if kt == RBF:
                kap = np.exp(-0.5 * s)
                psi = kap
            else:
                r = np.sqrt(np.maximum(s + 1e-20, 1e-20))
                if kt == M12:
                    a = np.maximum(-r, -20.0) if ard else -r
                    e = np.exp(a)
                    kap, psi = e, e / r
                elif kt == M32:
                    r3 = np.sqrt(3.0) * r
                    e = np.exp(np.maximum(-r3, -20.0))
                    kap, psi = (1.0 + r3) * e, 3.0 * e
                else:
                    r5 = np.sqrt(5.0) * r
                    e = np.exp(np.maximum(-r5, -20.0))
                    kap = (1.0 + r5 + 5.0 / 3.0 * s) * e
                    psi = 5.0 / 3.0 * (1.0 + r5) * e
            K = os * kap
        if want_grad:
            g = [None] * leaf_num_params(kt, ard, nd)
            if ard:
                for k in range(nd):
                    g[k] = os * psi * sq[:, :, k] / ell[k]
            else:
                g[0] = os * psi * s / p[0]
            g[os_idx] = kap
            if kt == RQ:
                g[nl] = g_alpha
            grads = g
        return K, grads
    if kt == PER:
        diff = X1[:, None, :] - X2[None, :, :]  # [n1, n2, nd]
        nl = nd if ard else 1
        period, os = p[nl], p[nl + 1]
        ell = p[:nd] if ard else np.full(nd, p[0])
        a = np.pi * diff / period
        sn, cs = np.sin(a), np.cos(a)
        arg = (sn * sn / ell).sum(axis=2)
        e = np.exp(-2.0 * arg)
        K = os * e
        if want_grad:
            g = [None] * (nl + 2)
            if ard:
                for k in range(nd):
                    g[k] = 2.0 * K * sn[:, :, k] ** 2 / ell[k] ** 2
            else:
                g[0] = 2.0 * K * arg / p[0]
            g[nl] = K * 4.0 * np.pi / period ** 2 * (sn * cs * diff / ell).sum(axis=2)
            g[nl + 1] = e
            grads = g
        return K, grads
    if kt == LIN:
        if ard:
            os = p[nd]
            dot = np.einsum("ik,jk,k->ij", X1, X2, p[:nd])
            K = os * dot
            if want_grad:
                grads = [os * np.outer(X1[:, k], X2[:, k]) for k in range(nd)] + [dot]
            return K, grads
        var, os = p[0], p[1]
        dot = X1 @ X2.T
        K = os * var * dot
        if want_grad:
            grads = [os * dot, var * dot]
        return K, grads
    if kt == POLY:
        bi = nd if ard else 0
        deg = int(round(p[bi]))
        off, os = p[bi + 1], p[bi + 2]
        dot = np.einsum("ik,jk,k->ij", X1, X2, p[:nd]) if ard else X1 @ X2.T
        base = dot + off
        K = os * base ** deg
        if want_grad:
            dbase = os * deg * base ** (deg - 1)
            g = [None] * (bi + 3)
            if ard:
                for k in range(nd):
                    g[k] = dbase * np.outer(X1[:, k], X2[:, k])
            g[bi] = np.zeros_like(K)
            g[bi + 1] = dbase
            g[bi + 2] = base ** deg
            grads = g
        return K, grads
    raise ValueError(kt)


def kernel_matrix(spec, params, X1, X2=None, want_grad=False):
    """K(X1, X2) in float64; with want_grad also the list of P dK/dtheta_p."""
    X1 = np.asarray(X1, dtype=np.float64)
    X1 = X1[:, None] if X1.ndim == 1 else X1
    X2 = X1 if X2 is None else np.asarray(X2, dtype=np.float64)
    X2 = X2[:, None] if X2.ndim == 1 else X2
    params = np.asarray(params, dtype=np.float64)
    P, nodes = parse(spec)
    stack = []  # entries: (K, {param_index: dK})
    for nd_ in nodes:
        if nd_[0] == "leaf":
            _, kt, ard, pofs, dims = nd_
            np_ = leaf_num_params(kt, ard, len(dims))
            K, g = _leaf(kt, ard, params[pofs:pofs + np_], X1[:, dims], X2[:, dims], want_grad)
            stack.append((K, {pofs + q: g[q] for q in range(np_)} if want_grad else {}))
        elif nd_[0] == "scale":
            K, g = stack.pop()
            c = params[nd_[1]]
            g2 = {q: c * v for q, v in g.items()}
            if want_grad:
                g2[nd_[1]] = K
            stack.append((c * K, g2))
        else:
            Kb, gb = stack.pop()
            Ka, ga = stack.pop()
            if nd_[0] == "sum":
                g = {**ga, **gb}
                stack.append((Ka + Kb, g))
            else:
                g = {q: v * Kb for q, v in ga.items()}
                g.update({q: Ka * v for q, v in gb.items()})
                stack.append((Ka * Kb, g))
    K, g = stack.pop()
    assert not stack
    if want_grad:
        return K, [g[q] for q in range(P)]
    return K


def forward_matvec(spec, params, X, V, noise=0.0, noise_vec=None, rows=None, block=1024):
    """(K + noise I) V in float64, V [n, t]; optionally only the given rows."""
    X = np.asarray(X, dtype=np.float64)
    X = X[:, None] if X.ndim == 1 else X
    V = np.asarray(V, dtype=np.float64)
    V2 = V[:, None] if V.ndim == 1 else V
    rows = np.arange(X.shape[0]) if rows is None else np.asarray(rows)
    out = np.empty((len(rows), V2.shape[1]))
    for b0 in range(0, len(rows), block):
        r = rows[b0:b0 + block]
        out[b0:b0 + block] = kernel_matrix(spec, params, X[r], X) @ V2
    nz = noise if noise_vec is None else np.asarray(noise_vec, dtype=np.float64)[rows][:, None]
    out += nz * V2[rows]
    return out[:, 0] if V.ndim == 1 else out


def cross_matvec(spec, params, Xtest, X, V, block=1024):
    Xtest = np.asarray(Xtest, dtype=np.float64)
    Xtest = Xtest[:, None] if Xtest.ndim == 1 else Xtest
    V = np.asarray(V, dtype=np.float64)
    V2 = V[:, None] if V.ndim == 1 else V
    out = np.empty((Xtest.shape[0], V2.shape[1]))
    for b0 in range(0, Xtest.shape[0], block):
        out[b0:b0 + block] = kernel_matrix(spec, params, Xtest[b0:b0 + block], X) @ V2
    return out[:, 0] if V.ndim == 1 else out


def gradient_bilinear(spec, params, X, A, B):
    """data[p] = a0' dK_p b0 ; trace[p] = sum_{c>=1} a_c' dK_p b_c (float64)."""
    _, G = kernel_matrix(spec, params, X, want_grad=True)
    A = np.asarray(A, np.float64)
    B = np.asarray(B, np.float64)
    data = np.array([A[:, 0] @ g @ B[:, 0] for g in G])
    trace = np.array([sum(A[:, c] @ g @ B[:, c] for c in range(1, A.shape[1])) for g in G])
    return data, trace


def gradient_bilinear_rows(spec, params, X, rows, A_rows, B, block=4):
    """gradient_bilinear restricted to rows: with a_i = 0 outside `rows`,
    data[p] = sum_{i in rows} a_i0 dK_p[i, :] b_0 and likewise trace over
    columns c >= 1. A_rows [len(rows), t] holds the nonzero rows of A. Row
    blocks keep memory at block x n x dims, so rows against 1e6 columns fit."""
    X = np.asarray(X, np.float64)
    B = np.asarray(B, np.float64)
    A_rows = np.asarray(A_rows, np.float64)
    rows = np.asarray(rows)
    data = trace = None
    for b0 in range(0, len(rows), block):
        r = rows[b0:b0 + block]
        _, G = kernel_matrix(spec, params, X[r], X, want_grad=True)
        a = A_rows[b0:b0 + block]
        d = np.array([a[:, 0] @ (g @ B[:, 0]) for g in G])
        t = np.array([np.sum(a[:, 1:] * (g @ B[:, 1:])) for g in G])
        data = d if data is None else data + d
        trace = t if trace is None else trace + t
    return data, trace
