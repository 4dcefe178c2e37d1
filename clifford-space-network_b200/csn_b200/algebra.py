"""Blade tables and real matrix representations for Cl(p, 0), and the code
generator for ``csrc/ga_tables.h``.

The reference multiplies blades by the bitmask rule of
``include/clifford_algebra.cuh:60-74``: the product of canonical blades e_a e_b
is ``(-1)^swaps e_{a xor b}`` where ``swaps`` counts pairs (i in a, j in b,
j < i); all basis vectors square to +1.  Reversion flips the sign of grades
with ``g(g-1)/2`` odd (``include/clifford_algebra.cuh:127-138``).  Blade orders
follow ``include/clifford_configs.cuh``: grade, then lexicographic, except that
the Cl(3,0) layout names its third bivector ``e31`` (= -e13)
(``include/clifford_configs.cuh:38-51``).

The reference's Cl(6)/Cl(8) code works with D x D real matrices
(``python/clifford_cl6.py:108-113``, ``python/clifford_cl8.py:132-135``).  To
feed blade-basis inputs into that matrix path this module builds a real
representation rho: Cl(n,0) -> M_D(R) in which every basis vector maps to a
symmetric signed-permutation matrix.  Then rho(reverse(a)) = rho(a)^T, every
bivector maps to a skew matrix, and the two-sided matrix scan
``X_t = M_t X_{t-1} M_t^T + C_t`` with ``M = rho(R)`` equals the blade-basis
recurrence ``h_t = R h_{t-1} R~ + x_t``.  Cl(3,0) -> M_4(R) and
Cl(8,0) -> M_16(R) (the latter an isomorphism).

Run ``python -m csn_b200.algebra`` (with the package directory on sys.path) to
regenerate ``csrc/ga_tables.h``.
"""
from __future__ import annotations

import itertools
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

__all__ = [
    "Algebra", "CL3", "CL4", "CL8", "real_rep", "bivector_basis", "triu_basis",
    "blades_to_matrix", "matrix_to_blades", "emit_header",
]


def _canon_sign(a: int, b: int) -> int:
    swaps = 0
    for i in range(16):
        if a >> i & 1:
            for j in range(i):
                if b >> j & 1:
                    swaps += 1
    return -1 if swaps & 1 else 1


def _popcount(x: int) -> int:
    return bin(x).count("1")


@dataclass
class Algebra:
    """Cl(n, 0) with an explicit blade order.

    ``masks[i]`` is the set of basis vectors of blade i, ``orient[i]`` = +-1 is
    its orientation relative to the increasing-index product.
    """
    n: int
    masks: list
    orient: list
    names: list
    prod_idx: np.ndarray = field(init=False)
    prod_sgn: np.ndarray = field(init=False)

    def __post_init__(self):
        nb = len(self.masks)
        where = {m: i for i, m in enumerate(self.masks)}
        self.prod_idx = np.zeros((nb, nb), dtype=np.int32)
        self.prod_sgn = np.zeros((nb, nb), dtype=np.int32)
        for i, j in itertools.product(range(nb), range(nb)):
            m = self.masks[i] ^ self.masks[j]
            k = where[m]
            self.prod_idx[i, j] = k
            self.prod_sgn[i, j] = (self.orient[i] * self.orient[j] * self.orient[k]
                                   * _canon_sign(self.masks[i], self.masks[j]))

    @property
    def size(self) -> int:
        return len(self.masks)

    def grade(self, i: int) -> int:
        return _popcount(self.masks[i])

    def rev_sign(self, i: int) -> int:
        g = self.grade(i)
        return -1 if (g * (g - 1) // 2) & 1 else 1

    def blades_of_grade(self, g: int) -> list:
        return [i for i in range(self.size) if self.grade(i) == g]

    def mul(self, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        """Geometric product over the last axis (numpy, any dtype)."""
        out = np.zeros(np.broadcast_shapes(a.shape, b.shape), dtype=np.result_type(a, b))
        for i, j in itertools.product(range(self.size), range(self.size)):
            out[..., self.prod_idx[i, j]] += self.prod_sgn[i, j] * a[..., i] * b[..., j]
        return out

    def reverse(self, a: np.ndarray) -> np.ndarray:
        s = np.array([self.rev_sign(i) for i in range(self.size)], dtype=a.dtype)
        return a * s


def _grade_lex(n: int):
    masks, names = [], []
    for g in range(n + 1):
        for combo in itertools.combinations(range(n), g):
            masks.append(sum(1 << c for c in combo))
            names.append("1" if g == 0 else "e" + "".join(str(c + 1) for c in combo))
    return masks, names


def _make_grade_lex(n: int) -> Algebra:
    masks, names = _grade_lex(n)
    return Algebra(n, masks, [1] * len(masks), names)


#: Cl(3,0) layout [1, e1, e2, e3, e12, e23, e31, e123] (include/clifford_configs.cuh:38-51)
CL3 = Algebra(3, [0, 1, 2, 4, 3, 6, 5, 7], [1, 1, 1, 1, 1, 1, -1, 1],
              ["1", "e1", "e2", "e3", "e12", "e23", "e31", "e123"])
#: Cl(4,0) layout of include/clifford_algebra.cuh:13-31 (grade, then lexicographic)
CL4 = _make_grade_lex(4)
#: Cl(8,0), 256 blades, grade then lexicographic; 28 bivectors e12 .. e78
CL8 = _make_grade_lex(8)

_I2 = np.eye(2)
_X2 = np.array([[0.0, 1.0], [1.0, 0.0]])
_Z2 = np.array([[1.0, 0.0], [0.0, -1.0]])
_J2 = np.array([[0.0, -1.0], [1.0, 0.0]])
_FACTORS = {"I": _I2, "X": _X2, "Z": _Z2, "J": _J2}
_ANTI = {frozenset("XZ"), frozenset("XJ"), frozenset("ZJ")}


def _kron(word: str) -> np.ndarray:
    m = np.ones((1, 1))
    for c in word:
        m = np.kron(m, _FACTORS[c])
    return m


def _anticommute(u: str, v: str) -> bool:
    return sum(frozenset((a, b)) in _ANTI for a, b in zip(u, v)) % 2 == 1


def _vector_words(n: int, k: int) -> list:
    """n mutually anticommuting symmetric words of k factors (even number of J)."""
    cands = ["".join(w) for w in itertools.product("IXZJ", repeat=k)
             if w.count("J") % 2 == 0 and any(c != "I" for c in w)]

    def search(chosen, start):
        if len(chosen) == n:
            return chosen
        for idx in range(start, len(cands)):
            w = cands[idx]
            if all(_anticommute(w, c) for c in chosen):
                r = search(chosen + [w], idx + 1)
                if r:
                    return r
        return None

    found = search([], 0)
    if found is None:
        raise ValueError(f"no real rep of Cl({n},0) on {2**k} dims from Kronecker words")
    return found


_REP_DIMS = {3: 2, 8: 4}  # Kronecker factors: Cl(3,0) -> M_4(R), Cl(8,0) -> M_16(R)


def real_rep(alg: Algebra) -> np.ndarray:
    """rho(blade_i) for every blade, shape [alg.size, D, D] (float64)."""
    k = _REP_DIMS[alg.n]
    vec = [_kron(w) for w in _vector_words(alg.n, k)]
    D = 2 ** k
    out = np.zeros((alg.size, D, D))
    for i, m in enumerate(alg.masks):
        mat = np.eye(D)
        for b in range(alg.n):
            if m >> b & 1:
                mat = mat @ vec[b]
        out[i] = alg.orient[i] * mat
    return out


def bivector_basis(alg: Algebra) -> np.ndarray:
    """E_k = rho(bivector_k) in the algebra's bivector order, [n(n-1)/2, D, D]."""
    rep = real_rep(alg)
    return rep[alg.blades_of_grade(2)]


def triu_basis(D: int) -> np.ndarray:
    """Skew basis of the reference generator layout (torch.triu_indices(D, D, 1)
    order, python/clifford_cl6.py:124-125, :155-158)."""
    iu, iv = np.triu_indices(D, 1)
    E = np.zeros((len(iu), D, D))
    E[np.arange(len(iu)), iu, iv] = 1.0
    E[np.arange(len(iu)), iv, iu] = -1.0
    return E


def blades_to_matrix(alg: Algebra, coeffs: np.ndarray) -> np.ndarray:
    """rho(sum_i c_i blade_i): [..., nblades] -> [..., D, D]."""
    rep = real_rep(alg)
    return np.einsum("...i,ijk->...jk", coeffs, rep)


def matrix_to_blades(alg: Algebra, mats: np.ndarray) -> np.ndarray:
    """Inverse of blades_to_matrix on the span of rho (trace inner product)."""
    rep = real_rep(alg)
    D = rep.shape[-1]
    return np.einsum("...jk,ijk->...i", mats, rep) / D


# ----------------------------------------------------------------- code generation
def _sandwich_poly(alg: Algebra, even: list):
    """L[i][j] as a quadratic form in the even rotor components:
    (R h R~)_i = sum_j sum_{a<=b} c[i][j][(a,b)] R_a R_b h_j."""
    nb = alg.size
    terms = {}
    for j in range(nb):
        for ai, a in enumerate(even):
            # e_a e_j
            k1 = alg.prod_idx[a, j]
            s1 = alg.prod_sgn[a, j]
            for bi, b in enumerate(even):
                # (e_a e_j) reverse(e_b)
                k2 = alg.prod_idx[k1, b]
                s2 = s1 * alg.prod_sgn[k1, b] * alg.rev_sign(b)
                key = (k2, j, min(ai, bi), max(ai, bi))
                terms[key] = terms.get(key, 0) + s2
    poly = {}
    for (i, j, a, b), c in terms.items():
        if c != 0:
            poly.setdefault((i, j), []).append((a, b, c))
    return poly


def _fmt_poly(entries, rv="r"):
    parts = []
    for a, b, c in sorted(entries):
        coef = "" if abs(c) == 1 else f"{float(abs(c))}f * "
        sign = "-" if c < 0 else "+"
        parts.append(f"{sign} {coef}{rv}{a} * {rv}{b}")
    s = " ".join(parts)
    return s[2:] if s.startswith("+ ") else s


def _fmt_unit_poly(entries, rv="r"):
    """L[i][j] for a unit rotor.  An entry with an r0^2 term is a number near 1 for the rotors
    of small steps; with r0^2 = 1 - r1^2 - r2^2 - r3^2 it is written as 1 + (small terms), the
    small part summed first, so the entry is rounded once, unbiased.  Summing the squares
    directly rounds quantities near 1 again and again, which leaves the map slightly
    contracting or expanding in the same direction every step."""
    c00 = sum(c for a, b, c in entries if a == 0 and b == 0)
    if c00 == 0:
        return _fmt_poly(entries, rv)
    rest = {}
    for a, b, c in entries:
        if a == 0 and b == 0:
            continue
        rest[(a, b)] = rest.get((a, b), 0) + c
    for m in (1, 2, 3):  # c00 r0^2 = c00 (1 - r1^2 - r2^2 - r3^2)
        rest[(m, m)] = rest.get((m, m), 0) - c00
    small = [(a, b, c) for (a, b), c in sorted(rest.items()) if c != 0]
    one = f"{float(c00)}f" if c00 != 1 else "1.0f"
    return f"{one} + ({_fmt_poly(small, rv)})" if small else one


def emit_header(path: Path) -> str:
    """Write csrc/ga_tables.h and return its text."""
    lines = [
        "// GENERATED by csn_b200/algebra.py -- do not edit by hand.",
        "// Blade tables and real representations for the rotor-scan kernels.",
        "#pragma once",
        "",
        "namespace csn {",
        "",
    ]
    # ---- Cl(3,0): rotor sandwich as an explicit linear map
    even = CL3.blades_of_grade(0) + CL3.blades_of_grade(2)  # [1, e12, e23, e31]
    poly = _sandwich_poly(CL3, even)
    lines += [
        "// Cl(3,0) blades [1, e1, e2, e3, e12, e23, e31, e123]; even rotor r = (r0, r1, r2, r3)",
        "// on [1, e12, e23, e31].  ga3_sandwich_matrix fills L with (R h R~) = L h.",
        "struct Ga3Map { float m[8][8]; };",
        "__host__ __device__ __forceinline__ void ga3_sandwich_matrix(float r0, float r1, float r2,",
        "                                                              float r3, Ga3Map& L) {",
        "#pragma unroll",
        "  for (int i = 0; i < 8; ++i)",
        "#pragma unroll",
        "    for (int j = 0; j < 8; ++j) L.m[i][j] = 0.0f;",
    ]
    nz = []
    for (i, j), ent in sorted(poly.items()):
        lines.append(f"  L.m[{i}][{j}] = {_fmt_unit_poly(ent)};")
        nz.append((i, j))
    lines += ["}", ""]
    # vector-Jacobian product of (R h R~) with respect to the rotor components:
    # dr_m = sum_ij G_i h_j dL_ij / dr_m, with L_ij a quadratic form in r
    lines += [
        "// dr[m] = sum_ij G[i] h[j] d(L[i][j]) / d r_m  (gradient of <G, R h R~> w.r.t. r)",
        "__host__ __device__ __forceinline__ void ga3_sandwich_vjp(float r0, float r1, float r2, float r3,",
        "                                                           const float h[8], const float G[8],",
        "                                                           float dr[4]) {",
        "  const float r[4] = {r0, r1, r2, r3};",
        "  float d0 = 0.0f, d1 = 0.0f, d2 = 0.0f, d3 = 0.0f;",
    ]
    acc = {m: [] for m in range(4)}
    for (i, j), ent in sorted(poly.items()):
        for a_, b_, c in ent:
            # d(c r_a r_b)/d r_m = c (delta_am r_b + delta_bm r_a)
            for m in range(4):
                k = (1 if a_ == m else 0) * 1 + (1 if b_ == m else 0) * 1
                if a_ == m and b_ == m:
                    acc[m].append((2 * c, a_, i, j))
                elif a_ == m:
                    acc[m].append((c, b_, i, j))
                elif b_ == m:
                    acc[m].append((c, a_, i, j))
    for m in range(4):
        for c, o, i, j in acc[m]:
            coef = f"{float(c)}f * " if abs(c) != 1 else ("-" if c < 0 else "")
            lines.append(f"  d{m} += {coef}r[{o}] * G[{i}] * h[{j}];")
    lines += ["  dr[0] = d0; dr[1] = d1; dr[2] = d2; dr[3] = d3;", "}", ""]
    lines.append("// nonzero pattern of the Cl(3,0) sandwich map (block diagonal by grade)")
    lines.append(f"#define CSN_GA3_NNZ {len(nz)}")
    lines.append("")
    # even product R2 R1 on [1, e12, e23, e31]
    lines += [
        "// product of two Cl(3,0) even elements a*b on [1, e12, e23, e31]",
        "__host__ __device__ __forceinline__ void ga3_even_mul(const float a[4], const float b[4],",
        "                                                       float out[4]) {",
    ]
    pos = {blade: p for p, blade in enumerate(even)}
    acc = {p: [] for p in range(4)}
    for pa, a in enumerate(even):
        for pb, b in enumerate(even):
            k = CL3.prod_idx[a, b]
            s = CL3.prod_sgn[a, b]
            acc[pos[k]].append(("-" if s < 0 else "+") + f" a[{pa}] * b[{pb}]")
    for p in range(4):
        e = " ".join(acc[p])
        e = e[2:] if e.startswith("+ ") else e
        lines.append(f"  out[{p}] = {e};")
    lines += ["}", ""]

    # ---- rho tables for generator bases (signed-permutation form)
    for alg, tag in ((CL3, "CL3"), (CL8, "CL8")):
        E = bivector_basis(alg)
        K, D, _ = E.shape
        cols = np.zeros((K, D), dtype=np.int32)
        sgns = np.zeros((K, D), dtype=np.int32)
        for k in range(K):
            for u in range(D):
                nzc = np.nonzero(E[k, u])[0]
                assert len(nzc) == 1, "rho(bivector) must be a signed permutation"
                cols[k, u] = nzc[0]
                sgns[k, u] = int(E[k, u, nzc[0]])
        lines.append(f"// rho(bivector_k) of {tag} as signed permutations: row u of rho(bivector_k)")
        lines.append("// has its one nonzero at column col[k][u] with sign sgn[k][u].  Use as a local")
        lines.append(f"// `constexpr auto t = {tag.lower()}_biv_tab();` so the tables fold into device code.")
        lines.append(f"#define CSN_{tag}_NBIV {K}")
        lines.append(f"#define CSN_{tag}_REPD {D}")
        lines.append(f"struct {tag.capitalize()}BivTab {{ unsigned char col[{K}][{D}]; signed char sgn[{K}][{D}]; }};")
        lines.append(f"__host__ __device__ constexpr {tag.capitalize()}BivTab {tag.lower()}_biv_tab() {{")
        lines.append(f"  return {tag.capitalize()}BivTab{{{{")
        for k in range(K):
            lines.append("    {" + ", ".join(str(int(c)) for c in cols[k]) + "},")
        lines.append("  }, {")
        for k in range(K):
            lines.append("    {" + ", ".join(str(int(x)) for x in sgns[k]) + "},")
        lines.append("  }};")
        lines.append("}")
        lines.append("")
    lines += ["}  // namespace csn", ""]
    text = "\n".join(lines)
    Path(path).write_text(text)
    return text


if __name__ == "__main__":
    out = Path(__file__).resolve().parent.parent / "csrc" / "ga_tables.h"
    emit_header(out)
    print(f"wrote {out}")
