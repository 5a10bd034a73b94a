"""Writes tests/golden/gguf_fuzz_corpus.json from the reference's FuzzParse corpus.

The reference fuzzes its GGUF header parser (gguf/gguf_test.go:80-85) and keeps
216 inputs in gguf/testdata/fuzz/FuzzParse/ (Go fuzz v1 text: one
``[]byte("...")`` line of a Go string literal). This script decodes each into
bytes and stores them as hex, so the parser tests can run where the reference
is not mounted. It only reads test inputs; it runs no reference code.

    python tests/golden/make_gguf_corpus.py /path/to/reference
"""

import json
import os
import sys


def go_unquote(lit: str) -> bytes:
    """Decodes a Go interpreted string literal (strconv.Quote's escapes) to bytes."""
    out = bytearray()
    i = 0
    simple = {"a": 7, "b": 8, "f": 12, "n": 10, "r": 13, "t": 9, "v": 11, "\\": 92, '"': 34, "'": 39}
    while i < len(lit):
        c = lit[i]
        if c != "\\":
            out += c.encode("utf-8")
            i += 1
            continue
        e = lit[i + 1]
        if e in simple:
            out.append(simple[e])
            i += 2
        elif e == "x":
            out.append(int(lit[i + 2:i + 4], 16))
            i += 4
        elif e == "u":
            out += chr(int(lit[i + 2:i + 6], 16)).encode("utf-8")
            i += 6
        elif e == "U":
            out += chr(int(lit[i + 2:i + 10], 16)).encode("utf-8", "surrogatepass")
            i += 10
        elif e in "01234567":
            out.append(int(lit[i + 1:i + 4], 8))
            i += 4
        else:
            raise ValueError(f"unknown escape \\{e}")
    return bytes(out)


def main(ref: str) -> None:
    d = os.path.join(ref, "gguf", "testdata", "fuzz", "FuzzParse")
    corpus = {}
    for name in sorted(os.listdir(d)):
        lines = open(os.path.join(d, name), encoding="utf-8").read().splitlines()
        assert lines[0] == "go test fuzz v1", name
        body = lines[1]
        assert body.startswith('[]byte("') and body.endswith('")'), name
        corpus[name] = go_unquote(body[len('[]byte("'):-2]).hex()
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "gguf_fuzz_corpus.json")
    with open(out, "w") as f:
        json.dump({"source": "gguf/testdata/fuzz/FuzzParse (go-wasmcontainers/llm)", "inputs": corpus}, f, indent=0,
                  sort_keys=True)
        f.write("\n")
    print(f"{len(corpus)} inputs -> {out}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_gguf_corpus.py REFERENCE_CHECKOUT")
    main(sys.argv[1])
