"""Packs the solution slot into solution/solution.json, the format the
contest harness builds from: config.toml's fields plus every source file
inlined, flat (kernel.cu, binding.py, the library's CUDA sources and its C
header), so that kernel.cu's includes resolve beside it.

    python solution/pack.py
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(ROOT, "karnbirkhera-mlsys2026-dsa_topk_indexer_b200", "csrc")
INCLUDE = os.path.join(ROOT, "include")
OUT = os.path.join(HERE, "solution.json")


def _toml(path):
    """The two tables of config.toml (flat key = value lines)."""
    out, table = {}, None
    for line in open(path):
        line = line.split("#", 1)[0].strip()
        if not line:
            continue
        if line.startswith("["):
            table = out.setdefault(line.strip("[]"), {})
        else:
            k, v = (x.strip() for x in line.split("=", 1))
            table[k] = {"true": True, "false": False}.get(v, v.strip('"'))
    return out


def sources():
    files = [os.path.join(HERE, "cuda", "kernel.cu"), os.path.join(HERE, "cuda", "binding.py")]
    files += [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cu", ".cuh", ".cc"))]
    files.append(os.path.join(INCLUDE, "dsa_topk_indexer.h"))
    return files


def pack():
    cfg = _toml(os.path.join(HERE, "config.toml"))
    sol, build = cfg["solution"], cfg["build"]
    doc = {
        "name": sol["name"],
        "definition": sol["definition"],
        "author": sol["author"],
        "spec": {
            "language": build["language"],
            "target_hardware": ["NVIDIA_B200"],
            "entry_point": build["entry_point"],
            "dependencies": [],
            "destination_passing_style": build["destination_passing_style"],
            "binding": build["binding"],
        },
        "sources": [{"path": os.path.basename(f), "content": open(f).read()} for f in sources()],
    }
    with open(OUT + ".tmp", "w") as f:
        json.dump(doc, f, indent=2)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(pack(), file=sys.stderr)
