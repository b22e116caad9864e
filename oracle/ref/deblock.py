"""Rewrite Apple block literals in the KERNIX reference headers into GNU C nested functions.

TEST INFRASTRUCTURE ONLY. This script is part of the recipe that compiles the reference's own
CPU forward (include/kernix.h, include/kernix_model.h, src/kernix_capi.c, src/kernix_runtime.c)
with gcc on Linux so that tests and the CPU-baseline leg of bench.py can run it. Its output goes to
oracle/_ref/ (git-ignored) and is never shipped or called by the product.

gcc has no Apple Blocks. Every block literal `^(params) { body }` in the reference headers is a
closure passed straight to a callee that calls it before returning (kernix_par, dispatch_apply,
kernix_matmul_ep_into's cpu_ep), so a GNU statement-expression nested function is an exact
stand-in: `({ void __kx_blkN(params) { body } __kx_blkN; })`. The two block typedefs
(include/kernix.h:385 kernix_range_fn, include/kernix.h:946 kernix_rows_fn) become plain function
pointer typedefs. Nothing else in the text changes.

usage: python deblock.py SRC_HEADER DST_HEADER
"""
import re
import sys


def _match_brace(src, i):
    """Index of the brace closing the one at src[i] (src[i] == '{'). Skips string/char literals and comments."""
    depth = 0
    k = i
    n = len(src)
    while k < n:
        c = src[k]
        if c == '"' or c == "'":
            q = c
            k += 1
            while k < n and src[k] != q:
                k += 2 if src[k] == "\\" else 1
        elif src.startswith("/*", k):
            k = src.index("*/", k) + 1
        elif src.startswith("//", k):
            k = src.index("\n", k)
        elif c == "{":
            depth += 1
        elif c == "}":
            depth -= 1
            if depth == 0:
                return k
        k += 1
    raise ValueError("unbalanced braces")


def deblock(src):
    src = re.sub(r"typedef\s+void\s*\(\^(\w+)\)", r"typedef void (*\1)", src)
    out = []
    i = 0
    count = 0
    while True:
        j = src.find("^(", i)
        if j < 0:
            out.append(src[i:])
            break
        close = src.index(")", j)
        params = src[j + 2:close]
        brace = src.index("{", close)
        if src[close + 1:brace].strip():
            raise ValueError(f"unexpected text between block parameters and body at offset {j}")
        end = _match_brace(src, brace)
        count += 1
        out.append(src[i:j])
        out.append(f"({{ void __kx_blk{count}({params}) {src[brace:end + 1]} __kx_blk{count}; }})")
        i = end + 1
    return "".join(out), count


if __name__ == "__main__":
    if len(sys.argv) != 3:
        sys.exit(__doc__)
    text, n = deblock(open(sys.argv[1], encoding="utf-8").read())
    with open(sys.argv[2], "w", encoding="utf-8") as f:
        f.write(text)
    print(f"{sys.argv[1]}: {n} block literals rewritten")
