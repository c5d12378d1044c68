r"""Generate csrc/unicode_tables.h from Python's unicodedata (the Unicode Character Database).

The byte-level BPE tokenizer (csrc/tokenizer.cpp) needs, for the GPT-2 style split and for
NFC normalisation:
  * ranges of general category L* (letters) and N* (numbers),
  * the White_Space property (PropList.txt; a fixed list, written out below),
  * word characters as regex `\w` defines them (UTS #18: Alphabetic, marks, decimal digits,
    connector punctuation, join controls), for added tokens with single_word,
  * canonical decompositions, canonical combining classes and the primary composites
    (pairs whose canonical composition is not excluded: NFC of the composite is itself).

The normalisation tables are pinned to the NFC of the reference's tokenizer library (HF
`tokenizers`, the version the reference's Cargo.lock pins) when its Python binding is
importable: that library's tables are of an older Unicode version, and it treats characters
assigned after it as starters without a decomposition. Each code point whose normalisation
differs between this unicodedata and the library (probed alone and next to combining marks)
is left out of the three tables, which makes libj1 treat it the same way.

Usage: python julia1-rs_b200/gen_unicode_tables.py   (rewrites csrc/unicode_tables.h)
"""
import os
import sys
import unicodedata

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "csrc", "unicode_tables.h")
MAXCP = 0x110000

# PropList.txt White_Space (unchanged since Unicode 6.3)
WHITE_SPACE = [(0x9, 0xD), (0x20, 0x20), (0x85, 0x85), (0xA0, 0xA0), (0x1680, 0x1680), (0x2000, 0x200A),
               (0x2028, 0x2029), (0x202F, 0x202F), (0x205F, 0x205F), (0x3000, 0x3000)]


# Other_Alphabetic code points outside L/M/Nl (PropList.txt): circled and squared Latin letters
OTHER_ALPHABETIC_SYMBOLS = [(0x24B6, 0x24E9), (0x1F130, 0x1F149), (0x1F150, 0x1F169), (0x1F170, 0x1F189)]


def is_word(cp):
    c = unicodedata.category(chr(cp))
    if c[0] in "LM" or c in ("Nd", "Nl", "Pc") or cp in (0x200C, 0x200D):
        return True
    return any(a <= cp <= b for a, b in OTHER_ALPHABETIC_SYMBOLS)


def ranges(pred):
    out, start = [], None
    for cp in range(MAXCP):
        if pred(cp):
            if start is None:
                start = cp
        elif start is not None:
            out.append((start, cp - 1))
            start = None
    if start is not None:
        out.append((start, MAXCP - 1))
    return out


def cat(cp):
    return unicodedata.category(chr(cp))


def canonical_decomposition(cp):
    d = unicodedata.decomposition(chr(cp))
    if not d or d.startswith("<"):
        return None
    return [int(x, 16) for x in d.split()]


def library_unknown():
    """Code points whose NFC/NFD differs between this unicodedata and the tokenizer
    library's normalizers, or (set(), None) when the library is not importable."""
    try:
        import tokenizers
        from tokenizers import normalizers
    except ImportError:
        return set(), None
    nfc, nfd = normalizers.NFC(), normalizers.NFD()
    out = set()
    for cp in range(MAXCP):
        if 0xD800 <= cp <= 0xDFFF:
            continue
        ch = chr(cp)
        d = unicodedata.decomposition(ch)
        if not unicodedata.combining(ch) and not (d and not d.startswith("<")):
            continue
        for s in (ch, "\u0345" + ch, "a" + ch + "\u0301", ch + "\u0301"):
            if nfd.normalize_str(s) != unicodedata.normalize("NFD", s) or \
                    nfc.normalize_str(s) != unicodedata.normalize("NFC", s):
                out.add(cp)
                break
    return out, tokenizers.__version__


def emit_ranges(name, rs):
    lines = ["constexpr uint32_t %s[][2] = {" % name]
    row = []
    for a, b in rs:
        row.append("{0x%X, 0x%X}" % (a, b))
        if len(row) == 6:
            lines.append("    " + ", ".join(row) + ",")
            row = []
    if row:
        lines.append("    " + ", ".join(row) + ",")
    lines.append("};")
    return lines


def main(out=OUT):
    letters = ranges(lambda cp: cat(cp).startswith("L"))
    numbers = ranges(lambda cp: cat(cp).startswith("N"))
    words = ranges(is_word)
    decomp, ccc, comp = [], [], []
    for cp in range(MAXCP):
        if 0xAC00 <= cp <= 0xD7A3:  # Hangul syllables: algorithmic
            continue
        c = unicodedata.combining(chr(cp))
        if c:
            ccc.append((cp, c))
        d = canonical_decomposition(cp)
        if d is not None:
            decomp.append((cp, d))
            if len(d) == 2 and unicodedata.normalize("NFC", chr(cp)) == chr(cp):
                comp.append((d[0], d[1], cp))
    comp.sort()
    unknown, lib_version = library_unknown()
    ccc = [x for x in ccc if x[0] not in unknown]
    decomp = [x for x in decomp if x[0] not in unknown]
    comp = [x for x in comp if not unknown.intersection(x)]
    pin = ("// Normalisation tables pinned to the NFC of HF tokenizers %s: %d code points newer than its"
           " Unicode tables are left out of them." % (lib_version, len(unknown))) if lib_version else \
        "// Normalisation tables not pinned (the tokenizer library was not importable)."
    L = ["// Generated by julia1-rs_b200/gen_unicode_tables.py from Python %s unicodedata (Unicode %s)."
         % (sys.version.split()[0], unicodedata.unidata_version), pin,
         "// Do not edit by hand.", "#pragma once", "#include <cstdint>", "", "namespace j1rt {", "namespace ucd {", "",
         "constexpr const char* kUnicodeVersion = \"%s\";" % unicodedata.unidata_version, ""]
    L += emit_ranges("kLetter", letters) + [""]
    L += emit_ranges("kNumber", numbers) + [""]
    L += emit_ranges("kWhiteSpace", WHITE_SPACE) + [""]
    L += emit_ranges("kWord", words) + [""]
    L.append("// canonical combining class != 0: {code point, class}")
    L.append("constexpr uint32_t kCombining[][2] = {")
    for i in range(0, len(ccc), 8):
        L.append("    " + ", ".join("{0x%X, %d}" % x for x in ccc[i:i + 8]) + ",")
    L.append("};")
    L.append("")
    L.append("// canonical decompositions (one level): {code point, first, second (0 if none)}")
    L.append("constexpr uint32_t kDecomposition[][3] = {")
    row = []
    for cp, d in decomp:
        assert len(d) in (1, 2), (hex(cp), d)
        row.append("{0x%X, 0x%X, 0x%X}" % (cp, d[0], d[1] if len(d) == 2 else 0))
        if len(row) == 5:
            L.append("    " + ", ".join(row) + ",")
            row = []
    if row:
        L.append("    " + ", ".join(row) + ",")
    L.append("};")
    L.append("")
    L.append("// primary composites, sorted by (first, second): {first, second, composite}")
    L.append("constexpr uint32_t kComposition[][3] = {")
    for i in range(0, len(comp), 5):
        L.append("    " + ", ".join("{0x%X, 0x%X, 0x%X}" % x for x in comp[i:i + 5]) + ",")
    L.append("};")
    L += ["", "}  // namespace ucd", "}  // namespace j1rt", ""]
    with open(out, "w") as f:
        f.write("\n".join(L))
    print("wrote %s: %d letter ranges, %d number ranges, %d combining, %d decompositions, %d compositions"
          % (out, len(letters), len(numbers), len(ccc), len(decomp), len(comp)))


if __name__ == "__main__":
    main()
