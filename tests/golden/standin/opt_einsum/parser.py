"""convert_to_valid_einsum_chars of the opt_einsum stand-in (see __init__.py)."""


def convert_to_valid_einsum_chars(einsum_str):
    symbols = sorted(set(einsum_str) - set(",->"))
    letters = "abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ"
    if len(symbols) > len(letters):
        raise ValueError("too many distinct einsum symbols")
    rename = {s: letters[k] for k, s in enumerate(symbols)}
    return "".join(rename.get(c, c) for c in einsum_str)
