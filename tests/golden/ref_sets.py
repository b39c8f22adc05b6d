"""Loader for the reference test-suite input sets (tests/golden/make_ref_sets.cpp).

The generator replays the reference's std::mt19937 draws with g++/libstdc++;
its outputs are pinned by the SHA-256 digests in ref_sets.sha256 (committed),
so a different standard library or a changed generator fails loudly rather
than silently testing different data. Regenerate the digest file with
`python tests/golden/ref_sets.py --write-digests`.
"""
from __future__ import annotations

import hashlib
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
GEN_SRC = HERE / "make_ref_sets.cpp"
OUT = HERE / "_gen"
DIGESTS = HERE / "ref_sets.sha256"


def generate() -> Path:
    OUT.mkdir(exist_ok=True)
    exe = OUT / "make_ref_sets"
    if not exe.exists() or exe.stat().st_mtime < GEN_SRC.stat().st_mtime:
        subprocess.run(["g++", "-O2", "-std=c++17", str(GEN_SRC), "-o", str(exe)], check=True)
        for f in OUT.glob("*.bin"):
            f.unlink()
    if not (OUT / "manifest.txt").exists() or not any(OUT.glob("*.bin")):
        subprocess.run([str(exe), str(OUT)], check=True)
    return OUT


def manifest() -> dict[str, int]:
    generate()
    out = {}
    for line in (OUT / "manifest.txt").read_text().split("\n"):
        if line.strip():
            name, u = line.split()
            out[name] = int(u)
    return out


def digests() -> dict[str, str]:
    out = {}
    for line in DIGESTS.read_text().split("\n"):
        if line.strip():
            d, name = line.split()
            out[name] = d
    return out


def load(name: str) -> tuple[np.ndarray, int]:
    """(bitset words u32, universe) of one set, digest-checked."""
    man = manifest()
    raw = (OUT / f"{name}.bin").read_bytes()
    want = digests().get(name)
    got = hashlib.sha256(raw).hexdigest()
    if want != got:
        raise AssertionError(f"reference set {name}: digest {got} != pinned {want}")
    return np.frombuffer(raw, dtype=np.uint32).copy(), man[name]


def ids_of(words: np.ndarray) -> np.ndarray:
    bits = np.unpackbits(words.view(np.uint8), bitorder="little")
    return np.flatnonzero(bits).astype(np.uint32)


if __name__ == "__main__":
    if "--write-digests" in sys.argv:
        man = manifest()
        lines = [f"{hashlib.sha256((OUT / f'{n}.bin').read_bytes()).hexdigest()} {n}" for n in man]
        DIGESTS.write_text("\n".join(lines) + "\n")
        print(f"wrote {len(lines)} digests")
