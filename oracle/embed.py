"""Write a C header holding the lines of a text file as a string array.

TEST INFRASTRUCTURE: the reference's cgen.c and fixer.c #include such headers
(rt_embed.h, rtq_embed.h, forest_embed.h); oracle/Makefile makes them here so
the reference compiles from its own sources into oracle/_ref/.
usage: embed.py ARRAY_NAME OUT.h [INPUT...]   (no input: an empty array)
"""
import sys


def main() -> None:
    name, out, inputs = sys.argv[1], sys.argv[2], sys.argv[3:]
    rows = [f"static const char *const {name}[] = {{"]
    for path in inputs:
        with open(path, encoding="utf-8") as f:
            for line in f.read().splitlines():
                esc = line.replace("\\", "\\\\").replace('"', '\\"')
                rows.append(f'\t"{esc}\\n",')
    rows.append("\t0\n};")
    with open(out, "w", encoding="utf-8") as f:
        f.write("\n".join(rows) + "\n")


if __name__ == "__main__":
    main()
