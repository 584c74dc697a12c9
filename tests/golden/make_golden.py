"""Regenerates the golden fixtures in this directory from the reference's own files.

    python tests/golden/make_golden.py REFERENCE_ROOT

Reads plain-text artifacts of rdadolf/ml-reentry-mlir from a checkout at
REFERENCE_ROOT (required) and writes small .npz files; nothing at test time
reads the reference tree. Fixtures:

  gcn_toy.npz       conv1/conv2 weights and biases of the GCN toy model, decoded
                    from the dense_resource blobs of test/reference/gcn.raw.mlir:26-35
                    (4-byte alignment header, then little-endian float32).
  gat_toy.npz       lin / att_src / att_dst of GATConv(4, 2, heads=2) from
                    experiments/gatconv/dumps/gat.1-raw-torch.mlir:137-139.
  sage_toy.npz      lin_l weight / bias and lin_r weight of the two SAGEConv layers of
                    the SAGE toy model, from test/reference/sage.raw.mlir:35-40.
  kat_softmax.npz   the 64x32 output of the row-max / exp-sum / weighted-aggregate
                    probe, parsed from experiments/gat-gpu-codegen/dumps/cpu.out.txt.
  kat_spmm.npz      the 8x8 and 8x4 SpMM outputs of
                    experiments/sparsifier-coo-check/dumps/{01-spmm-csr,05-spmm-weighted-csr}.out.txt.
  csr_small.npz     torch's coalesce -> to_sparse_csr of gcn_norm-normalised small
                    graphs with duplicate edges and self-loops (the reference's
                    normalized_csr_adj, gnnc/examples/util.py:16-41, run here with
                    torch; gcn_norm restated as in oracle/gnn_oracle.py).
"""

from __future__ import annotations

import re
import struct
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import gnn_oracle as O  # noqa: E402


def _resources(path: Path) -> dict[str, np.ndarray]:
    out = {}
    for name, hexs in re.findall(r'(torch_tensor_[\w.]+): "0x([0-9A-F]+)"', path.read_text()):
        raw = bytes.fromhex(hexs)
        assert struct.unpack("<I", raw[:4])[0] == 4, "expected a 4-byte alignment header"
        out[name] = np.frombuffer(raw[4:], dtype="<f4").copy()
    return out


def _memref(path: Path) -> np.ndarray:
    text = path.read_text()
    shape = [int(v) for v in re.search(r"sizes = \[([\d, ]+)\]", text).group(1).split(",")]
    body = text[text.index("data =") + len("data =") :]
    vals = [float(v) for v in re.findall(r"-?\d+(?:\.\d+)?(?:e[-+]?\d+)?", body)]
    return np.array(vals, dtype=np.float64).reshape(shape)


def main(root: Path) -> None:
    r = _resources(root / "test/reference/gcn.raw.mlir")
    np.savez(
        HERE / "gcn_toy.npz",
        w1=r["torch_tensor_8_4_torch.float32"].reshape(8, 4),
        b1=r["torch_tensor_8_torch.float32"],
        w2=r["torch_tensor_3_8_torch.float32"].reshape(3, 8),
        b2=r["torch_tensor_3_torch.float32"],
    )
    g = _resources(root / "experiments/gatconv/dumps/gat.1-raw-torch.mlir")
    np.savez(
        HERE / "gat_toy.npz",
        lin=g["torch_tensor_4_4_torch.float32"].reshape(4, 4),
        att_src=g["torch_tensor_1_2_2_torch.float32"].reshape(1, 2, 2),
        att_dst=g["torch_tensor_1_2_2_torch.float32_1"].reshape(1, 2, 2),
        edge_index=np.array([[0, 1, 0], [1, 2, 2]], dtype=np.int64),
    )
    sg = _resources(root / "test/reference/sage.raw.mlir")
    np.savez(
        HERE / "sage_toy.npz",
        wl1=sg["torch_tensor_8_4_torch.float32"].reshape(8, 4),
        bl1=sg["torch_tensor_8_torch.float32"],
        wr1=sg["torch_tensor_8_4_torch.float32_1"].reshape(8, 4),
        wl2=sg["torch_tensor_3_8_torch.float32"].reshape(3, 8),
        bl2=sg["torch_tensor_3_torch.float32"],
        wr2=sg["torch_tensor_3_8_torch.float32_1"].reshape(3, 8),
    )
    np.savez(HERE / "kat_softmax.npz",
             y=_memref(root / "experiments/gat-gpu-codegen/dumps/cpu.out.txt"))
    d = root / "experiments/sparsifier-coo-check/dumps"
    np.savez(HERE / "kat_spmm.npz", y01=_memref(d / "01-spmm-csr.out.txt"),
             y05=_memref(d / "05-spmm-weighted-csr.out.txt"))

    # Small graphs with duplicates and existing self-loops; CSR via torch coalesce.
    graphs = {}
    gen = torch.Generator().manual_seed(1234)
    for i, (n, e) in enumerate([(5, 12), (17, 60), (64, 400), (300, 3000)]):
        ei = torch.randint(0, n, (2, e), generator=gen)
        ei = torch.cat([ei, ei[:, : e // 5]], dim=1)  # duplicates
        crow, col, val = O.normalized_csr_adj(ei, n)
        graphs[f"g{i}_n"] = np.array(n)
        graphs[f"g{i}_edge_index"] = ei.numpy()
        graphs[f"g{i}_crow"] = crow.numpy()
        graphs[f"g{i}_col"] = col.numpy()
        graphs[f"g{i}_val"] = val.numpy()
    ring = torch.stack([torch.arange(5), (torch.arange(5) + 1) % 5])
    crow, col, val = O.normalized_csr_adj(ring, 5)
    graphs.update(ring_crow=crow.numpy(), ring_col=col.numpy(), ring_val=val.numpy())
    np.savez(HERE / "csr_small.npz", **graphs)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py REFERENCE_ROOT (a checkout of rdadolf/ml-reentry-mlir)")
    main(Path(sys.argv[1]))
