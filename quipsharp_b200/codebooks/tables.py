"""Exact construction of the two 256x8 codebook tables, in integer arithmetic.

Both tables are returned doubled (every entry x2, so all entries are integers);
divide by two for the real values.  The construction restates:

* E8P base table -- quipsharp/codebooks/e8p.py:64-89: the distinct
  elementwise-|x| patterns of D8-hat = {x in Z^8 + 1/2 : sum(x) even} with
  ||x||^2 <= 10 in lexicographic order (the order `torch.unique(dim=0)`
  returns), then the 29 padding rows of e8p.py:31-61, then the last coordinate
  of every odd-sum row is negated (e8p.py:75-81).
* 1-bit E8 table -- quipsharp/codebooks/e8_1bit.py:52-71: the zero row, the
  240 norm^2=2 vectors (integer ones then half-integer ones, each in
  cartesian-product order), then the first 15 integer norm^2=4 vectors.

This module has no torch dependency: the native build step imports it to bake
the tables into the CUDA library, and the codebook classes expose the same
rows as torch tensors.
"""
from __future__ import annotations

import itertools

CODE_DIM = 8

PAD29_X2 = (
    (3, 1, 1, 1, 3, 3, 3, 3), (1, 3, 1, 1, 3, 3, 3, 3), (1, 1, 3, 1, 3, 3, 3, 3),
    (1, 1, 1, 3, 3, 3, 3, 3), (3, 3, 3, 1, 3, 3, 1, 1), (3, 3, 3, 1, 3, 1, 3, 1),
    (3, 3, 3, 1, 1, 3, 3, 1), (3, 3, 3, 1, 3, 1, 1, 3), (3, 3, 3, 1, 1, 3, 1, 3),
    (3, 3, 3, 1, 1, 1, 3, 3), (3, 3, 1, 3, 3, 3, 1, 1), (3, 3, 1, 3, 3, 1, 3, 1),
    (3, 3, 1, 3, 1, 3, 3, 1), (3, 3, 1, 3, 3, 1, 1, 3), (3, 3, 1, 3, 1, 3, 1, 3),
    (3, 3, 1, 3, 1, 1, 3, 3), (3, 1, 3, 3, 3, 3, 1, 1), (3, 1, 3, 3, 3, 1, 3, 1),
    (3, 1, 3, 3, 1, 3, 3, 1), (3, 1, 3, 3, 3, 1, 1, 3), (3, 1, 3, 3, 1, 3, 1, 3),
    (1, 3, 3, 3, 1, 1, 3, 3), (1, 3, 3, 3, 3, 3, 1, 1), (1, 3, 3, 3, 3, 1, 3, 1),
    (1, 3, 3, 3, 1, 3, 3, 1), (1, 3, 3, 3, 3, 1, 1, 3), (1, 3, 3, 3, 1, 3, 1, 3),
    (1, 1, 3, 3, 1, 3, 3, 3), (3, 3, 1, 1, 3, 3, 3, 1),
)


def d8hat_abs_patterns_x2():
    """The 227 |x| patterns (x2) of D8-hat inside the ball ||x||^2 <= 10.

    Flipping one coordinate of a half-integer vector changes its sum by an odd
    integer, so every half-integer |x| pattern has an even-sum signing: the
    patterns are exactly the half-integer vectors of the positive orthant in
    the ball, sorted lexicographically."""
    rows = [r for r in itertools.product((1, 3, 5, 7), repeat=CODE_DIM)
            if sum(v * v for v in r) <= 40]
    rows.sort()
    assert len(rows) == 227
    return rows


def e8p_abs_table_x2():
    rows = [list(r) for r in d8hat_abs_patterns_x2()] + [list(r) for r in PAD29_X2]
    assert len(rows) == 256
    for r in rows:
        if (sum(r) // 2) % 2 != 0:          # sum(x) = sum(2x)/2; odd -> negate last coordinate
            r[-1] = -r[-1]
    return [tuple(r) for r in rows]


def _int_shell_x2(norm_sq):
    b = int(norm_sq ** 0.5)
    return [tuple(2 * v for v in r) for r in itertools.product(range(-b, b + 1), repeat=CODE_DIM)
            if sum(v * v for v in r) == norm_sq and sum(r) % 2 == 0]


def _half_shell_x2(norm_sq):
    b = int(norm_sq ** 0.5) + 1
    vals2 = [2 * v + 1 for v in range(-b, b)]
    return [r for r in itertools.product(vals2, repeat=CODE_DIM)
            if sum(v * v for v in r) == 4 * norm_sq and (sum(r) // 2) % 2 == 0]


def e8_1bit_table_x2():
    shell = _int_shell_x2(2) + _half_shell_x2(2)
    assert len(shell) == 240
    table = [(0,) * CODE_DIM] + shell + _int_shell_x2(4)[:15]
    assert len(table) == 256 and len(set(table)) == 256
    return table
