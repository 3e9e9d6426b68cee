"""Build and run the native ``genesis-pack`` corpus packer (``csrc/tools/genesis_pack.cpp``).

``build_genesis_pack()`` compiles the tool with the host C++ compiler into
``llm_research_b200/bin/genesis-pack`` (rebuilt when the source is newer);
``pack_corpus(...)`` runs it and returns the parsed ``meta.json``.  The
output layout matches the reference tool (``data_tools/src/main.rs``):
``train_input_ids.bin`` / ``val_input_ids.bin`` (little-endian uint32 blocks)
and ``meta.json``; :class:`~olympus.data.packed_dataset.PackedDataset` reads it.
"""

from __future__ import annotations

import json
import os
import shutil
import subprocess
from typing import Any, Dict, Optional

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
SOURCE = os.path.join(_ROOT, "csrc", "tools", "genesis_pack.cpp")
BINARY = os.path.join(_ROOT, "llm_research_b200", "bin", "genesis-pack")


def build_genesis_pack(force: bool = False) -> str:
    deps = [SOURCE, os.path.join(os.path.dirname(SOURCE), "unicode_tables.h")]
    if not force and os.path.exists(BINARY) and all(os.path.getmtime(BINARY) >= os.path.getmtime(d) for d in deps):
        return BINARY
    cxx = os.environ.get("CXX") or shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("no C++ compiler found to build genesis-pack")
    os.makedirs(os.path.dirname(BINARY), exist_ok=True)
    tmp = BINARY + ".tmp"
    subprocess.run([cxx, "-O3", "-std=c++17", "-pthread", SOURCE, "-o", tmp], check=True)
    os.replace(tmp, BINARY)
    return BINARY


def pack_corpus(input_dir: str, output_dir: str, vocab: str, block_size: int = 4096, train_ratio: float = 0.98,
                eos_id: int = 100279, threads: Optional[int] = None) -> Dict[str, Any]:
    exe = build_genesis_pack()
    cmd = [exe, "--input-dir", input_dir, "--output-dir", output_dir, "--vocab", vocab, "--block-size",
           str(block_size), "--train-ratio", repr(float(train_ratio)), "--eos-id", str(eos_id)]
    if threads:
        cmd += ["--threads", str(threads)]
    subprocess.run(cmd, check=True, stdout=subprocess.DEVNULL)
    with open(os.path.join(output_dir, "meta.json")) as f:
        return json.load(f)
