"""Independent restatement of the DPA4C-style (se_e2_a type) model in PyTorch.

Used only to generate and check golden fixtures: forces and virials come from
autograd, the neighbour list from a brute-force image enumeration, so nothing
here shares code with the C++ oracle (oracle/sea_oracle.cpp) or the CUDA path.
Same conventions: neighbours of i are (j, n) with r = x'_j + n.B - x'_i,
|r| < rcut; per type sorted by (r^2, j, image code), first sel[t] kept.
"""
from __future__ import annotations

import math

import numpy as np
import torch


def image_code(n0, n1, n2):
    return ((n0 + 512) << 20) | ((n1 + 512) << 10) | (n2 + 512)


def box_inverse(box):
    B = np.asarray(box, dtype=np.float64).reshape(3, 3)
    return np.linalg.inv(B)


def brute_nlist(coord, atype, box, rcut, sel, ntypes):
    """Periodic neighbour list by enumerating every image within reach."""
    coord = np.asarray(coord, np.float64)
    B = np.asarray(box, np.float64).reshape(3, 3)
    Binv = box_inverse(B)
    s = coord @ Binv
    f = np.floor(s)
    xw = coord - (f[:, :1] * B[0] + f[:, 1:2] * B[1] + f[:, 2:3] * B[2])
    vol = abs(np.linalg.det(B))
    widths = [vol / np.linalg.norm(np.cross(B[(d + 1) % 3], B[(d + 2) % 3])) for d in range(3)]
    reach = [int(math.ceil(rcut / w)) + 1 for w in widths]
    n = coord.shape[0]
    selt = int(sum(sel))
    off = np.concatenate([[0], np.cumsum(sel)])
    nl = -np.ones((n, selt), np.int64)
    img = np.zeros((n, selt, 3), np.int64)
    rc2 = rcut * rcut
    shifts = []
    for a in range(-reach[0], reach[0] + 1):
        for b in range(-reach[1], reach[1] + 1):
            for c in range(-reach[2], reach[2] + 1):
                shifts.append((a, b, c))
    shifts = np.array(shifts)
    svec = shifts[:, :1] * B[0] + shifts[:, 1:2] * B[1] + shifts[:, 2:3] * B[2]
    for i in range(n):
        cands = [[] for _ in range(ntypes)]
        for si, (sh, sv) in enumerate(zip(shifts, svec)):
            r = (xw + sv) - xw[i]
            r2 = (r[:, 0] * r[:, 0] + r[:, 1] * r[:, 1]) + r[:, 2] * r[:, 2]
            for j in np.nonzero(r2 < rc2)[0]:
                if j == i and not sh.any():
                    continue
                cands[atype[j]].append((r2[j], int(j), image_code(*sh), tuple(sh)))
        for t in range(ntypes):
            c = sorted(cands[t], key=lambda q: (q[0], q[1], q[2]))[: sel[t]]
            for k, q in enumerate(c):
                nl[i, off[t] + k] = q[1]
                img[i, off[t] + k] = q[3]
    return nl, img, xw


def energy_torch(model, xw, atype, box, nl, img):
    """Energy of the formatted list; xw is a leaf tensor (wrapped coordinates)."""
    B = torch.as_tensor(np.asarray(box).reshape(3, 3), dtype=torch.float64)
    n, selt = nl.shape
    off = np.concatenate([[0], np.cumsum(model.sel)])
    valid = nl >= 0
    jj = torch.as_tensor(np.where(valid, nl, 0))
    shift = torch.as_tensor(img, dtype=torch.float64) @ B
    r = xw[jj] + shift - xw[:, None, :]
    r = torch.where(torch.as_tensor(valid)[..., None], r, torch.ones_like(r))
    rr = torch.sqrt((r * r).sum(-1))
    rs, rc = model.rcut_smth, model.rcut
    u = (rr - rs) / (rc - rs)
    sw = torch.where(rr < rs, torch.ones_like(rr),
                     torch.where(rr < rc, u ** 3 * (-6 * u ** 2 + 15 * u - 10) + 1, torch.zeros_like(rr)))
    vmask = torch.as_tensor(valid, dtype=torch.float64)
    s = sw / rr * vmask
    rt = torch.stack([s, s * r[..., 0] / rr, s * r[..., 1] / rr, s * r[..., 2] / rr], -1)
    M1 = model.emb[-1]
    T = torch.zeros(n, 4, M1, dtype=torch.float64)
    for t in range(model.ntypes):
        sl = slice(off[t], off[t + 1])
        for ti in range(model.ntypes):
            rows = torch.as_tensor(np.nonzero(np.asarray(atype[:n]) == ti)[0])
            if len(rows) == 0:
                continue
            net = model.emb_nets[t if model.type_one_side else ti * model.ntypes + t]
            x = s[rows][:, sl].reshape(-1, 1)
            for (w, b) in net:
                w = torch.as_tensor(w)
                b = torch.as_tensor(b)
                h = torch.tanh(x @ w + b)
                if w.shape[1] == w.shape[0]:
                    x = x + h
                elif w.shape[1] == 2 * w.shape[0]:
                    x = torch.cat([x, x], 1) + h
                else:
                    x = h
            G = x.reshape(len(rows), off[t + 1] - off[t], M1)
            G = G * vmask[rows][:, sl, None]
            T = T.index_add(0, rows, torch.einsum("nsk,nsa->nka", rt[rows][:, sl], G))
    T = T / float(selt)
    D = torch.einsum("nka,nkb->nab", T, T[:, :, : model.axis]).reshape(n, -1)
    E = torch.zeros(n, dtype=torch.float64)
    for ti in range(model.ntypes):
        rows = torch.as_tensor(np.nonzero(np.asarray(atype[:n]) == ti)[0])
        if len(rows) == 0:
            continue
        x = D[rows]
        net = model.fit_nets[ti]
        for l, (w, b) in enumerate(net):
            w = torch.as_tensor(w)
            b = torch.as_tensor(b)
            if l == len(net) - 1:
                x = x @ w + b
            else:
                h = torch.tanh(x @ w + b)
                x = x + h if (l >= 1 and w.shape[0] == w.shape[1]) else h
        E = E.index_put((rows,), x[:, 0] + model.bias_atom_e[ti])
    return E, r, D


def evaluate(model, coord, atype, box):
    nl, img, xw_np = brute_nlist(coord, atype, box, model.rcut, model.sel, model.ntypes)
    xw = torch.tensor(xw_np, requires_grad=True)
    E, r, D = energy_torch(model, xw, atype, box, nl, img)
    etot = E.sum()
    gx, gr = torch.autograd.grad(etot, [xw, r], retain_graph=False)
    valid = torch.as_tensor(nl >= 0)[..., None]
    gr = torch.where(valid, gr, torch.zeros_like(gr))
    r = r.detach()
    vir = -torch.einsum("nsa,nsb->ab", gr, r)
    n = coord.shape[0]
    av = torch.zeros(n, 9, dtype=torch.float64)
    jj = torch.as_tensor(np.where(nl >= 0, nl, 0))
    contrib = (-gr[..., :, None] * r[..., None, :]).reshape(n, -1, 9) * valid
    av = av.index_add(0, jj.reshape(-1), contrib.reshape(-1, 9))
    return dict(energy=float(etot.detach()), force=(-gx).numpy(), virial=vir.numpy(), atom_energy=E.detach().numpy(),
                atom_virial=av.numpy(), nlist=nl, image=img, descriptor=D.detach().numpy())
