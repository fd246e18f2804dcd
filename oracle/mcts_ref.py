"""AlphaZero search and xiangqi move rules restated - TEST INFRASTRUCTURE ONLY.

`legal_moves` restates Position's move rules (src/xiangqi/mod.rs: general and
advisor inside the palace, elephant eye and river, horse leg, rook slides,
cannon screens, soldier after the river, no move that leaves the mover's
general attacked or facing the other general) in plain Python.  `Search`
restates AzTree (src/az/alphazero.rs:959-1817) for one root at a time - the
reference's single-tree path: root expansion, then per simulation the PUCT
descent (compute_cpuct :1718-1739, FPU reduction :1795-1817, ties by prior),
leaf evaluation by the oracle's C evaluator (refresh, value head, threat
logits, policy logits), softmax priors, forced-reply extension, backup with
WDL flips - to check the wide-batch GPU search against.
"""
from __future__ import annotations

import math

import numpy as np

from . import (az_dense_moves, az_features, az_policy_logits, az_policy_moves, az_policy_refresh, az_quantize,
               az_refresh, az_threat_features, az_threat_logits, az_value)

F = np.float32


def _color(v):
    return 0 if v > 0 else 1


def _kind(v):
    return abs(int(v)) - 1


def _on(f, r):
    return 0 <= f < 9 and 0 <= r < 10


def _palace(c, f, r):
    return 3 <= f <= 5 and (7 <= r <= 9 if c == 0 else 0 <= r <= 2)


def _own_half(c, r):
    return r >= 5 if c == 0 else r <= 4


def pseudo_moves(b, side):
    out = []
    for sq in range(90):
        v = int(b[sq])
        if v == 0 or _color(v) != side:
            continue
        f, r = sq % 9, sq // 9
        k = _kind(v)
        targets = []
        if k == 0:
            targets = [(f + dx, r + dy) for dx, dy in ((1, 0), (-1, 0), (0, 1), (0, -1)) if _palace(side, f + dx, r + dy)]
        elif k == 1:
            targets = [(f + dx, r + dy) for dx, dy in ((1, 1), (1, -1), (-1, 1), (-1, -1)) if _palace(side, f + dx, r + dy)]
        elif k == 2:
            for dx, dy in ((2, 2), (2, -2), (-2, 2), (-2, -2)):
                if _on(f + dx, r + dy) and _own_half(side, r + dy) and b[(r + dy // 2) * 9 + f + dx // 2] == 0:
                    targets.append((f + dx, r + dy))
        elif k == 3:
            # HORSE_STEPS order (src/xiangqi/mod.rs:2140-2149)
            for dx, dy in ((-1, -2), (1, -2), (-1, 2), (1, 2), (-2, -1), (-2, 1), (2, -1), (2, 1)):
                leg = (f, r + dy // 2) if abs(dy) == 2 else (f + dx // 2, r)
                if _on(f + dx, r + dy) and b[leg[1] * 9 + leg[0]] == 0:
                    targets.append((f + dx, r + dy))
        elif k in (4, 5):
            for dx, dy in ((1, 0), (-1, 0), (0, 1), (0, -1)):
                tf, tr, screen = f + dx, r + dy, False
                while _on(tf, tr):
                    t = int(b[tr * 9 + tf])
                    if k == 4:
                        targets.append((tf, tr))
                        if t != 0:
                            break
                    elif not screen:
                        if t == 0:
                            targets.append((tf, tr))
                        else:
                            screen = True
                    elif t != 0:
                        targets.append((tf, tr))
                        break
                    tf, tr = tf + dx, tr + dy
        else:
            fwd = -1 if side == 0 else 1
            targets.append((f, r + fwd))
            if not _own_half(side, r):
                targets += [(f - 1, r), (f + 1, r)]
        for tf, tr in targets:
            if not _on(tf, tr):
                continue
            t = int(b[tr * 9 + tf])
            if t != 0 and (_color(t) == side or _kind(t) == 0):  # own piece, or any general
                continue
            out.append((sq, tr * 9 + tf))
    return out


def _checkers(b, g, by):
    """Pieces of `by` whose move pattern reaches g, plus a facing general."""
    n = 0
    for sq in range(90):
        v = int(b[sq])
        if v == 0 or _color(v) != by:
            continue
        c = np.array(b, np.int8)
        c[g] = -int(np.sign(v)) * 2  # a capturable stand-in for the general
        if (sq, g) in pseudo_moves(c, by):
            n += 1
    h = _general(b, by)
    if h >= 0 and h % 9 == g % 9:
        lo, hi = sorted((h // 9, g // 9))
        n += all(b[rr * 9 + g % 9] == 0 for rr in range(lo + 1, hi))
    return n


def _general(b, c):
    for sq in range(90):
        if b[sq] != 0 and _color(b[sq]) == c and _kind(b[sq]) == 0:
            return sq
    return -1


def _attacked(b, sq, by):
    """Every pseudo move of `by` that lands on sq, plus the facing generals."""
    c = np.array(b, np.int8)
    if c[sq] != 0 and _kind(c[sq]) == 0:
        c[sq] = -int(np.sign(c[sq])) * -2  # stand-in advisor of the owner: capturable, not a general
    for frm, to in pseudo_moves(c, by):
        if to == sq:
            return True
    g = _general(b, by)
    if g >= 0 and g % 9 == sq % 9:
        lo, hi = sorted((g // 9, sq // 9))
        if all(b[rr * 9 + sq % 9] == 0 for rr in range(lo + 1, hi)):
            return True
    return False


def legal_moves(b, side):
    """Position::legal_moves order: square order; in check by one piece the
    general's moves first."""
    pseudo = pseudo_moves(b, side)
    g = _general(b, side)
    if g >= 0 and _attacked(b, g, 1 - side) and _checkers(b, g, 1 - side) == 1:
        pseudo = [m for m in pseudo if m[0] == g] + [m for m in pseudo if m[0] != g]
    out = []
    for frm, to in pseudo:
        c = np.array(b, np.int8)
        c[to], c[frm] = c[frm], 0
        g = _general(c, side)
        if g < 0 or not _attacked(c, g, 1 - side):
            out.append((frm, to))
    return out


def searchable_moves(b, side, s2d):
    """Legal moves whose canonical move lies in the 2086-move policy space."""
    out = []
    for frm, to in legal_moves(b, side):
        cf, ct = (frm, to) if side == 0 else (89 - frm, 89 - to)
        if s2d[cf * 90 + ct] != 0xFFFF:
            out.append((frm, to))
    return out


def in_check(b, side):
    g = _general(b, side)
    return g >= 0 and _attacked(b, g, 1 - side)


class Evaluator:
    """One leaf at a time through the oracle's C restatement of the evaluator."""

    def __init__(self, tensors, hidden, threat_active, tactical_active):
        self.t, self.h = tensors, hidden
        self.quant = az_quantize(tensors, hidden)
        self.threat, self.tactical = threat_active, tactical_active

    def __call__(self, board, side, moves, rule):
        items = az_features(board, side)
        offs = np.array([0, len(items)], np.uint32)
        _, acc = az_refresh(self.t, self.h, items, offs)
        _, pacc = az_policy_refresh(self.quant["policy_feature"], items, offs)
        tl = act = None
        if self.threat:
            tf = az_threat_features(board, side)
            _, tl, act = az_threat_logits(self.quant["value_threat"], float(self.quant["scales"][3]), self.t[11], tf,
                                          np.array([0, len(tf)], np.uint32), with_act=True)
        wdl, q, x = az_value(self.t, self.h, acc, None if rule is None else rule[None], tl, with_x=True)
        info = az_policy_moves(board, side, np.array(moves, np.uint8).reshape(-1, 2)).astype(np.uint32)
        logits = az_policy_logits(self.t, self.h, self.quant, self.tactical, x, act, pacc, info,
                                  np.array([0, len(moves)], np.uint32))
        return wdl[0].astype(F), F(q[0]), np.asarray(logits[:len(moves)], F)


def _utility(wdl, draw):
    return F(min(max(F(F(wdl[0] - wdl[2]) + F(draw * wdl[1])), F(-1)), F(1)))


def _sum_utility(s, visits, draw):
    if visits == 0:
        return F(0)
    v = F(visits)
    return _utility([F(s[0] / v), F(s[1] / v), F(s[2] / v)], draw)


class Search:
    """AzTree for one root (defaults of AzSearchLimits)."""

    def __init__(self, evaluator, board, side, sims, rule=None, cpuct=1.5, base=19652.0, factor=2.0, fpu=0.30,
                 fpu_root=0.20, temp=1.0, draw=0.0):
        self.ev, self.sims, self.rule = evaluator, sims, rule
        self.cpuct, self.base, self.factor, self.fpu, self.fpu_root = F(cpuct), F(base), F(factor), F(fpu), F(fpu_root)
        self.temp, self.draw = F(temp), F(draw)
        self.nodes = [dict(board=np.array(board, np.int8), side=side, children=None, visits=0, wsum=[F(0)] * 3,
                           value=F(0), wdl=[F(0), F(1), F(0)], expanded=False)]
        self.s2d = np.full(8100, 0xFFFF, np.int64)
        self.s2d[az_dense_moves().astype(np.int64)] = np.arange(2086)

    def _terminal(self, n):
        kinds = [(_color(v), _kind(v)) for v in n["board"] if v != 0]
        if (0, 0) not in kinds:
            return F(-1) if n["side"] == 0 else F(1)
        if (1, 0) not in kinds:
            return F(-1) if n["side"] == 1 else F(1)
        return None

    def _expand(self, ni, moves, logits):
        mx = max(logits)
        inv = F(1) / max(self.temp, F(1e-3))
        pr = [F(np.exp(F(F(l - mx) * inv))) for l in logits]
        s = F(0)
        for p in pr:
            s = F(s + p)
        inv_s = F(1) / max(s, F(1e-12))
        self.nodes[ni]["children"] = [dict(mv=m, prior=F(p * inv_s), visits=0, wsum=[F(0)] * 3, node=None)
                                      for m, p in zip(moves, pr)]
        self.nodes[ni]["expanded"] = True

    def _eval_leaf(self, ni, moves):
        n = self.nodes[ni]
        wdl, q, logits = self.ev(n["board"], n["side"], moves, self.rule)
        n["value"], n["wdl"] = q, list(wdl)
        return list(wdl), q, logits

    def _child(self, ni, ci):
        c = self.nodes[ni]["children"][ci]
        if c["node"] is None:
            b = self.nodes[ni]["board"].copy()
            frm, to = c["mv"]
            b[to], b[frm] = b[frm], 0
            self.nodes.append(dict(board=b, side=1 - self.nodes[ni]["side"], children=None, visits=0,
                                   wsum=[F(0)] * 3, value=F(0), wdl=[F(0), F(1), F(0)], expanded=False))
            c["node"] = len(self.nodes) - 1
        return c["node"]

    def _draw(self, ni):
        return self.draw if self.nodes[ni]["side"] == self.nodes[0]["side"] else -self.draw

    def _select(self, ni):
        n = self.nodes[ni]
        root = ni == 0
        draw = self._draw(ni)
        psq = F(math.sqrt(F(max(n["visits"], 1))))
        pq = _sum_utility(n["wsum"], n["visits"], draw) if n["visits"] > 0 else _utility(n["wdl"], draw)
        red = self.fpu_root if root else self.fpu
        fpu = pq
        if red > 0:
            vis = F(0)
            for c in n["children"]:
                if c["visits"] > 0:
                    vis = F(vis + max(c["prior"], F(0)))
            vis = min(max(vis, F(0)), F(1))
            fpu = F(min(max(F(pq - F(red * F(math.sqrt(vis)))), F(-1)), F(1)))
        c_ = F(self.cpuct + F(self.factor * F(math.log(F(F(F(n["visits"]) + self.base) / self.base)))))
        best, bs, bp = None, None, None
        for i, c in enumerate(n["children"]):
            q = _sum_utility(c["wsum"], c["visits"], draw) if c["visits"] > 0 else fpu
            u = F(F(F(c_ * c["prior"]) * psq) / F(F(1) + F(c["visits"])))
            sc = F(q + u)
            if best is None or sc > bs or (sc == bs and c["prior"] > bp):
                best, bs, bp = i, sc, c["prior"]
        return best

    def _finish(self, path, node, wdl, value):
        n = self.nodes[node]
        n["visits"] += 1
        n["wsum"] = [F(a + b) for a, b in zip(n["wsum"], wdl)]
        for pi, ci in reversed(path):
            wdl = [wdl[2], wdl[1], wdl[0]]
            c = self.nodes[pi]["children"][ci]
            c["visits"] += 1
            c["wsum"] = [F(a + b) for a, b in zip(c["wsum"], wdl)]
            p = self.nodes[pi]
            p["visits"] += 1
            p["wsum"] = [F(a + b) for a, b in zip(p["wsum"], wdl)]

    def run(self):
        root = self.nodes[0]
        t = self._terminal(root)
        if t is not None:
            root["value"], root["expanded"], root["children"] = t, True, []
        else:
            moves = searchable_moves(root["board"], root["side"], self.s2d)
            if not moves:
                root["value"], root["wdl"], root["expanded"], root["children"] = F(-1), [F(0), F(0), F(1)], True, []
            else:
                _, _, logits = self._eval_leaf(0, moves)
                self._expand(0, moves, logits)
        max_depth = self.sims
        done = 0
        while done < self.sims:
            node, depth, path = 0, 0, []
            while True:
                n = self.nodes[node]
                cutoff = depth >= max_depth
                if cutoff and n["expanded"]:
                    self._finish(path, node, n["wdl"], n["value"])
                    break
                if cutoff or not n["expanded"]:
                    t = self._terminal(n)
                    if t is not None:
                        wdl = [F(1), F(0), F(0)] if t > 0 else ([F(0), F(0), F(1)] if t < 0 else [F(0), F(1), F(0)])
                        n["value"], n["wdl"] = t, wdl
                        if not cutoff:
                            n["expanded"], n["children"] = True, []
                        self._finish(path, node, wdl, t)
                        break
                    moves = searchable_moves(n["board"], n["side"], self.s2d)
                    if not moves:
                        n["value"], n["wdl"] = F(-1), [F(0), F(0), F(1)]
                        if not cutoff:
                            n["expanded"], n["children"] = True, []
                        self._finish(path, node, n["wdl"], n["value"])
                        break
                    check = (not cutoff) and in_check(n["board"], n["side"])
                    wdl, q, logits = self._eval_leaf(node, moves)
                    if cutoff:
                        self._finish(path, node, wdl, q)
                        break
                    self._expand(node, moves, logits)
                    if check or len(moves) == 1:
                        child = self._child(node, 0)
                        path.append((node, 0))
                        node, depth = child, depth + 1
                        continue
                    self._finish(path, node, wdl, q)
                    break
                if not n["children"]:
                    self._finish(path, node, n["wdl"], n["value"])
                    break
                ci = self._select(node)
                child = self._child(node, ci)
                path.append((node, ci))
                node, depth = child, depth + 1
            done += 1
        return self

    def result(self):
        ch = self.nodes[0]["children"] or []
        return {"moves": [c["mv"] for c in ch], "visits": [c["visits"] for c in ch],
                "priors": [float(c["prior"]) for c in ch]}
