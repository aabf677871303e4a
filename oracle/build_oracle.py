"""Build the C part of the CPU oracle (TEST INFRASTRUCTURE ONLY).

    python oracle/build_oracle.py

Compiles oracle/sampler_oracle.c into oracle/_build/liboracle.so with IEEE-strict flags
(-ffp-contract=off, no fast-math) so its float operations happen exactly in source order.
"""
import pathlib
import subprocess

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "_build" / "liboracle.so"
SRC = [HERE / "sampler_oracle.c"]


def build(force=False):
    OUT.parent.mkdir(exist_ok=True)
    newest = max(p.stat().st_mtime for p in SRC + [pathlib.Path(__file__)])
    if OUT.exists() and not force and OUT.stat().st_mtime >= newest:
        return OUT
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
           "-std=c11", *map(str, SRC), "-o", str(OUT), "-lm"]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force=True))
