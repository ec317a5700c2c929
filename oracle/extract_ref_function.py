"""Copy one function of a reference source file, as it lies, into oracle/_ref/ for compiling.

TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline). src/sparse.cpp of the
reference project defines trellis::build_neighbor_table with plain STL, but the same file
includes ggml headers for its graph builders, and ggml is absent, so the file as a whole cannot
be compiled. This script writes the function's own text, unchanged, between the standard headers
it uses and its namespace, into a file under oracle/_ref/ (git-ignored, never committed), which
the Makefile compiles next to oracle/ref_nbr.cpp.

usage: extract_ref_function.py <source.cpp> <signature prefix> <namespace> <out.cpp>
"""
import sys


def extract(src: str, prefix: str) -> str:
    start = src.index(prefix)
    depth, i, opened = 0, start, False
    while i < len(src):
        ch = src[i]
        if ch == "{":
            depth += 1
            opened = True
        elif ch == "}":
            depth -= 1
            if opened and depth == 0:
                return src[start:i + 1]
        i += 1
    raise ValueError("unbalanced braces after " + prefix)


def main():
    path, prefix, ns, out = sys.argv[1:5]
    body = extract(open(path).read(), prefix)
    with open(out, "w") as f:
        f.write("// extracted at build time from " + path + "; not part of this repository\n")
        f.write("#include <array>\n#include <cstdint>\n#include <unordered_map>\n#include <vector>\n")
        f.write("namespace " + ns + " {\n" + body + "\n}  // namespace " + ns + "\n")


if __name__ == "__main__":
    main()
