"""Minimal stand-in for the third-party `opt_einsum` package (not installed here, not vendored by the reference),
written for tests/golden/make_golden.py only, so the reference modules import and run on the CPU.

The reference uses three names (psgd_pro.py:16, :172-238; psgd_pro_fast.py:26):
  get_symbol(i)                 the i-th einsum index symbol (opt_einsum's published mapping: 52 ASCII letters,
                                then chr(i + 140), skipping the surrogate block)
  contract_expression(s, *shp)  a callable that evaluates the einsum `s` on operands of those shapes
  parser.convert_to_valid_einsum_chars(s)   rename every symbol to an ASCII letter torch.einsum accepts
The contraction runs as one torch.einsum call, so its order (and last-bit rounding) differs from opt_einsum's
greedy path; results agree with opt_einsum to fp32 rounding, which the golden tolerances allow for."""
from . import parser

_BASE = "abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ"


def get_symbol(i):
    if i < 52:
        return _BASE[i]
    if i >= 55296:
        return chr(i + 2048)
    return chr(i + 140)


class ContractExpression:
    """Evaluates the einsum by greedy pairwise contraction: at each step the pair of operands whose intermediate
    result is smallest is contracted (one torch.einsum per pair), as opt_einsum's greedy strategy does."""

    def __init__(self, subscripts, shapes):
        self.subscripts = subscripts
        self.shapes = shapes
        eq = parser.convert_to_valid_einsum_chars(subscripts)
        self._inputs, self._output = eq.split("->")[0].split(","), eq.split("->")[1]

    def __call__(self, *operands):
        import torch
        terms = list(zip(self._inputs, operands))
        size = {}
        for idx, op in terms:
            for c, n in zip(idx, op.shape):
                size[c] = n
        while len(terms) > 1:
            best = None
            for i in range(len(terms)):
                for j in range(i + 1, len(terms)):
                    rest = "".join(t[0] for k, t in enumerate(terms) if k not in (i, j)) + self._output
                    keep = "".join(dict.fromkeys(c for c in terms[i][0] + terms[j][0] if c in rest))
                    shared = set(terms[i][0]) & set(terms[j][0])
                    cost = 1
                    for c in keep:
                        cost *= size[c]
                    key = (0 if shared else 1, cost)
                    if best is None or key < best[0]:
                        best = (key, i, j, keep)
            _, i, j, keep = best
            (si, a), (sj, b) = terms[i], terms[j]
            res = torch.einsum(f"{si},{sj}->{keep}", a, b)
            terms = [t for k, t in enumerate(terms) if k not in (i, j)] + [(keep, res)]
        idx, res = terms[0]
        return torch.einsum(f"{idx}->{self._output}", res) if idx != self._output else res


def contract_expression(subscripts, *shapes, **kwargs):
    return ContractExpression(subscripts, shapes)
