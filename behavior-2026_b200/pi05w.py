"""Weight files of the pi0.5 engine (.pi05w): read, write, and convert between the engine's own layout
and the reference engine's layout.

The format is the reference's (docs/archive/windows/π05_네이티브엔진.md:46-49): a text manifest --
"pi05w 1", "cfg <key> <value>" lines with the model hyper-parameters, "t <name> <bf16|f32> <offset>
<bytes> <dims...>" lines, "end" -- padded to 256 bytes, then the raw tensors at 256-byte aligned offsets.
Every linear layer is stored [out][in].

Two tensor layouts load (pi05_load_weights accepts either, tensor by tensor):
  engine     what pi05_save_weights writes: fused q|k|v per layer, gate/up rows interleaved ("gu.w", row
             2j = gate j, 2j+1 = up j), the SigLIP patch embedding padded to 640 columns, the adaRMS
             modulation Denses stacked ("exp.ada.w"), bf16;
  reference  the reference exporter's conventions: separate q / k / v and gate / up tensors (the
             engine interleaves gate/up rows, and q/k rows per head for its fused RoPE, when it loads),
             the SigLIP MLP padded 4304 -> 4352 with zeros (dropped on load), the patch embedding at its
             588 columns ((ky * 14 + kx) * 3 + channel), one modulation Dense per norm
             ("exp.l<N>.ada1/ada2", "exp.final.ada"), f32 as exported from the f32 checkpoint (rounded
             to bf16 on load).
`to_reference_layout` converts the first to the second; `main` writes a seeded synthetic checkpoint in
the reference layout (the engine's pi05_init_random_weights weights, which need a GPU).
"""
import argparse
import os

import numpy as np

CFG_KEYS = ("siglip_layers", "gemma_layers", "expert_layers", "num_steps", "n_cameras", "n_text", "horizon")
SIG_MLP, SIG_MLP_PAD, SIG_K, QD, HD = 4304, 4352, 588, 2048, 256


def _bf16_to_f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def _f32_to_bf16(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def read(path):
    """(cfg {key: int}, {name: float32 array of the stored dims}); bf16 tensors are widened exactly"""
    with open(path, "rb") as f:
        lines, size = [], 0
        while True:
            line = f.readline()
            if not line:
                raise ValueError("truncated manifest")
            size += len(line)
            text = line.decode().rstrip("\n")
            if text == "end":
                break
            lines.append(text)
        hdr = (size + 255) & ~255
        if not lines or not lines[0].startswith("pi05w"):
            raise ValueError("not a pi05w file")
        cfg, tensors = {}, {}
        for text in lines[1:]:
            p = text.split()
            if p[0] == "cfg":
                cfg[p[1]] = int(p[2])
            elif p[0] == "t":
                name, dt, off, nbytes, dims = p[1], p[2], int(p[3]), int(p[4]), [int(d) for d in p[5:]]
                f.seek(hdr + off)
                raw = f.read(nbytes)
                a = np.frombuffer(raw, np.float32 if dt == "f32" else np.uint16)
                a = a.copy() if dt == "f32" else _bf16_to_f32(a)
                tensors[name] = a.reshape(dims)
    return cfg, tensors


def write(path, cfg, tensors, dtype="f32"):
    """tensors {name: array}; stored as `dtype` (bf16 values are rounded to nearest even)"""
    es = 4 if dtype == "f32" else 2
    man, off, blobs = ["pi05w 1"] + [f"cfg {k} {cfg[k]}" for k in CFG_KEYS if k in cfg], 0, []
    for name, a in tensors.items():
        a = np.asarray(a, np.float32)
        raw = (a if dtype == "f32" else _f32_to_bf16(a)).tobytes()
        assert len(raw) == a.size * es
        man.append(f"t {name} {dtype} {off} {len(raw)} " + " ".join(str(d) for d in a.shape))
        blobs.append((off, raw))
        off += (len(raw) + 255) & ~255
    text = ("\n".join(man) + "\nend\n").encode()
    hdr = (len(text) + 255) & ~255
    with open(path, "wb") as f:
        f.write(text + b"\n" * (hdr - len(text)))
        for at, raw in blobs:
            f.seek(hdr + at)
            f.write(raw)
        f.truncate(hdr + off)


def to_reference_layout(cfg, tensors):
    """engine layout -> the reference exporter's layout (see the module docstring)"""
    out = {}
    for name, a in tensors.items():
        parts = name.split(".")
        base = ".".join(parts[:-2]) + "." if len(parts) > 2 else ""
        if name.endswith(".qkv.w") or name.endswith(".qkv.b"):
            sig = name.startswith("sig.")
            fq, fk = (1152, 1152) if sig else (QD, HD)
            kind = name[-1]
            flat = a if kind == "w" else a.reshape(-1)
            q, k, v = flat[:fq], flat[fq:fq + fk], flat[fq + fk:fq + 2 * fk]
            out[base + "q." + kind], out[base + "k." + kind], out[base + "v." + kind] = q, k, v
        elif name.endswith(".gu.w"):
            out[base + "gate.w"], out[base + "up.w"] = a[0::2], a[1::2]
        elif name.startswith("sig.") and name.endswith(".mlp1.w"):
            out[name] = np.concatenate([a, np.zeros((SIG_MLP_PAD - SIG_MLP, a.shape[1]), np.float32)], 0)
        elif name.startswith("sig.") and name.endswith(".mlp1.b"):
            flat = a.reshape(-1)
            out[name] = np.concatenate([flat, np.zeros(SIG_MLP_PAD - SIG_MLP, np.float32)])
        elif name.startswith("sig.") and name.endswith(".mlp2.w"):
            out[name] = np.concatenate([a, np.zeros((a.shape[0], SIG_MLP_PAD - SIG_MLP), np.float32)], 1)
        elif name == "sig.stem.w":
            out[name] = np.ascontiguousarray(a[:, :SIG_K])
        elif name in ("exp.ada.w", "exp.ada.b"):
            nm = 2 * cfg["expert_layers"] + 1
            per = a.reshape(nm, 3 * 1024, -1) if name.endswith("w") else a.reshape(nm, 3 * 1024)
            for m in range(nm):
                key = "exp.final.ada" if m == nm - 1 else f"exp.l{m // 2}.ada{m % 2 + 1}"
                out[key + name[-2:]] = per[m]
        else:
            out[name] = a
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description="write a seeded synthetic pi0.5 checkpoint in the reference layout")
    ap.add_argument("--out", required=True)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--siglip-layers", type=int, default=27)
    ap.add_argument("--gemma-layers", type=int, default=18)
    ap.add_argument("--num-steps", type=int, default=10)
    ap.add_argument("--dtype", default="f32", choices=["f32", "bf16"])
    args = ap.parse_args(argv)
    import pi05native as pn

    eng = pn.Engine(pn.Config.make(siglip_layers=args.siglip_layers, gemma_layers=args.gemma_layers,
                                   num_steps=args.num_steps), max_batch=1)
    eng.init_random_weights(args.seed)
    tmp = args.out + ".engine-layout"
    eng.save_weights(tmp)
    eng.close()
    cfg, tensors = read(tmp)
    os.remove(tmp)
    write(args.out, cfg, to_reference_layout(cfg, tensors), args.dtype)


if __name__ == "__main__":
    main()
