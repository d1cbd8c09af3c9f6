"""Helpers shared by the GPU parity tests."""
import numpy as np

TOL_FP32 = 1e-4                 # rel-L2, fp32 features
TOL_FP16 = (1e-3, 1e-2)         # rel-L2, max-abs, fp16 / bf16 / Q8_0 features


def dev(a, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(t):
    import torch
    return t.detach().float().cpu().numpy() if t.dtype != torch.int32 else t.cpu().numpy()


def q8_blocks(oracle, w):
    """ggml block_q8_0 rows of w as a raw uint8 array (34 bytes per 32 values)."""
    q = oracle.quantize_q8_0(np.asarray(w, dtype=np.float32))
    return np.frombuffer(q.tobytes(), dtype=np.uint8).copy()


def weight_tensor(oracle, w, wtype):
    import torch
    if wtype == "f32":
        return dev(np.asarray(w, dtype=np.float32))
    if wtype == "f16":
        return dev(np.asarray(w, dtype=np.float32)).to(torch.float16)
    return dev(q8_blocks(oracle, w))


def numpy_neighbor_map(coords):
    """Independent neighbour map by sorted-key search (no hash)."""
    from mogecpp_b200.synth import pack_keys
    n = coords.shape[0]
    keys = pack_keys(coords)
    order = np.argsort(keys, kind="stable")
    sk = keys[order]
    out = np.empty((n, 27), dtype=np.int32)
    v = 0
    c64 = coords.astype(np.int64)
    for dx in (-1, 0, 1):
        for dy in (-1, 0, 1):
            for dz in (-1, 0, 1):
                q = c64.copy()
                q[:, 0] += dx
                q[:, 1] += dy
                q[:, 2] += dz
                ok = np.all((q[:, :3] >= 0) & (q[:, :3] < (1 << 19)), axis=1)
                qk = pack_keys(np.where(ok[:, None], q, 0))
                pos = np.minimum(np.searchsorted(sk, qk), n - 1)
                hit = ok & (sk[pos] == qk)
                out[:, v] = np.where(hit, order[pos], n)
                v += 1
    return out
