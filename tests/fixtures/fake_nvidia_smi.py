#!/usr/bin/env python3
"""Fake nvidia-smi for topology tests: FAKE_GPU_MEM="183359,183359,..." (MiB per GPU), FAKE_LINK=NV18|PIX."""
import os
import sys

mem = [int(x) for x in os.environ.get("FAKE_GPU_MEM", ",".join(["183359"] * 8)).split(",")]
link = os.environ.get("FAKE_LINK", "NV18")
args = sys.argv[1:]
if args and args[0].startswith("--query-gpu"):
    for i, m in enumerate(mem):
        print(f"{i}, {m}")
elif args[:2] == ["topo", "-m"]:
    n = len(mem)
    print("\t" + "\t".join(f"GPU{i}" for i in range(n)) + "\tCPU Affinity")
    for i in range(n):
        row = ["X" if i == j else link for j in range(n)]
        print(f"GPU{i}\t" + "\t".join(row) + "\t0-111")
else:
    sys.exit(1)
