"""Write reference cases in the upstream data layout, for its benchmark scripts.

    python fast-cuda-cross-attention_b200/make_reference_data.py --config c3 --out data
    python fast-cuda-cross-attention_b200/make_reference_data.py --config c4 --out data
    python fast-cuda-cross-attention_b200/make_reference_data.py --config c5 --out data

Each case is a directory holding Q_matrix.npy, K_matrix.npy, V_matrix.npy (float32,
[B, N, D]; [N, D] for the single-batch cases, as upstream's generate_references.py writes
them) and output_reference.npy (float32, [B, N_latent, D]) -- the files upstream's
benchmark.py / benchmark_batching.py read (benchmark.py:71-84) -- plus meta.json:

    c1, c2   data/N_latent_{Nl}                      B=1, N_input=784 (upstream layout)
    c3       data/batches/batch_{B}/N_latent_{Nl}    B in 4..32, N_input=784 (upstream layout)
    c4       data/config4                            B=8, Nl=512, Ni=65536, K,V ~ N(0, 0.5^2)
    c5       data/config5                            bf16 multi-head B=32, H=8, d=96

Inputs follow the upstream generators' seeding (np.random.seed(42), then Q, K, V from
randn in that order; config 4 scales K and V by 0.5).  Config 5 stores the bf16-rounded
values as float32 (exact; .npy has no bf16 type).  The reference output is computed in
float64 on the GPU (torch, in row chunks), so it is independent of this library's kernels.
Before writing, the free space of --out is checked against the case's size (config 4 is
3.2 GB of inputs); too little space refuses with an error instead of a partial write.
"""

import argparse
import json
import math
import os
import shutil
import sys

import numpy as np

CASES = {
    "c1": [dict(b=1, nl=64, ni=784, single=True)],
    "c2": [dict(b=1, nl=nl, ni=784, single=True) for nl in (64, 128, 256, 512, 1024)],
    "c3": [dict(b=b, nl=nl, ni=784) for b in (4, 8, 16, 32) for nl in (64, 128, 256, 512, 1024)],
    "c4": [dict(b=8, nl=512, ni=65536, kv_std=0.5)],
    "c5": [dict(b=32, nl=1024, ni=784, heads=8)],
}
D = 768


def case_dir(out, config, c):
    if config in ("c1", "c2"):
        return os.path.join(out, f"N_latent_{c['nl']}")
    if config == "c3":
        return os.path.join(out, "batches", f"batch_{c['b']}", f"N_latent_{c['nl']}")
    return os.path.join(out, "config4" if config == "c4" else "config5")


def case_bytes(c):
    return 4 * (2 * c["b"] * c["nl"] * D + 2 * c["b"] * c["ni"] * D)  # Q, K, V, output


def reference(q, k, v, heads, device):
    """float64 softmax(q k^T / sqrt(d)) v per head, row chunks bounded to ~1 GB of scores."""
    import torch

    b, nl, dm = q.shape
    dh = dm // heads
    out = np.empty((b, nl, dm), dtype=np.float32)
    rows = max(1, int(1.25e8 // max(1, k.shape[1])))
    for i in range(b):
        kk = torch.from_numpy(k[i]).to(device, torch.float64)
        vv = torch.from_numpy(v[i]).to(device, torch.float64)
        for h in range(heads):
            kh, vh = kk[:, h * dh:(h + 1) * dh], vv[:, h * dh:(h + 1) * dh]
            for r0 in range(0, nl, rows):
                qh = torch.from_numpy(q[i, r0:r0 + rows, h * dh:(h + 1) * dh]).to(device, torch.float64)
                o = torch.softmax(qh @ kh.T / math.sqrt(dh), -1) @ vh
                out[i, r0:r0 + rows, h * dh:(h + 1) * dh] = o.cpu().numpy()
    return out


def write_case(path, c, device):
    np.random.seed(42)  # upstream: np.random.seed(seed), then Q, K, V
    q = np.random.randn(c["b"], c["nl"], D).astype(np.float32)
    k = np.random.randn(c["b"], c["ni"], D).astype(np.float32)
    v = np.random.randn(c["b"], c["ni"], D).astype(np.float32)
    if "kv_std" in c:
        k *= np.float32(c["kv_std"])
        v *= np.float32(c["kv_std"])
    heads = c.get("heads", 1)
    if heads > 1:  # bf16-rounded inputs, kept as float32
        import torch

        q, k, v = (torch.from_numpy(x).bfloat16().float().numpy() for x in (q, k, v))
    ref = reference(q, k, v, heads, device)  # [B, Nl, D]
    if c.get("single"):  # upstream single-batch files: 2-D inputs, [1, Nl, D] output
        q, k, v = q[0], k[0], v[0]
    os.makedirs(path, exist_ok=True)
    for name, arr in (("Q_matrix", q), ("K_matrix", k), ("V_matrix", v), ("output_reference", ref)):
        np.save(os.path.join(path, f"{name}.npy"), arr)
    with open(os.path.join(path, "meta.json"), "w") as f:
        json.dump(dict(B=c["b"], N_latent=c["nl"], N_input=c["ni"], D=D, heads=heads,
                       kv_std=c.get("kv_std", 1.0), seed=42,
                       dtype="bf16-rounded float32" if heads > 1 else "float32",
                       reference="float64 torch, softmax(q k^T / sqrt(d)) v per head"), f, indent=1)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", choices=sorted(CASES), required=True)
    ap.add_argument("--out", default="data")
    ap.add_argument("--device", default="cuda")
    a = ap.parse_args(argv)
    cases = CASES[a.config]
    need = sum(case_bytes(c) for c in cases)
    os.makedirs(a.out, exist_ok=True)
    free = shutil.disk_usage(a.out).free
    if free < need * 1.1:
        raise SystemExit(f"{a.config}: needs {need / 1e9:.2f} GB in {a.out}, {free / 1e9:.2f} GB free")
    for c in cases:
        path = case_dir(a.out, a.config, c)
        write_case(path, c, a.device)
        print(f"wrote {path}")


if __name__ == "__main__":
    sys.exit(main())
