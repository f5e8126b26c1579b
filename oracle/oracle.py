"""ctypes wrapper of the CPU oracle (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, and only to check results or time the CPU baseline. It wraps oracle/_build/libkgoracle.so, a C++
restatement of katgpt-rs's x86-64 AVX2 forward path (see kg_oracle.h).

Parity pin: partial. The reference has no golden files and cannot be built
here (Rust); the oracle is pinned to the reference's own test assertions and
invariants (tests/test_oracle.py, tests/test_paged_oracle.py,
tests/test_sq_oracle.py) and, to three or four significant digits, to two of
its published benchmark tables (TurboQuant and SpectralQuant reconstruction
quality on seeded keys), not to bit-exact reference outputs.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBPATH = os.path.join(HERE, "_build", "libkgoracle.so")

MODE_BASE, MODE_QUANT, MODE_SPKV, MODE_QUANT_AS_WRITTEN = 0, 1, 2, 3


class OrConfig(ctypes.Structure):
    _fields_ = [("vocab_size", ctypes.c_int32), ("block_size", ctypes.c_int32),
                ("n_embd", ctypes.c_int32), ("n_head", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("n_kv_head", ctypes.c_int32),
                ("mlp_hidden", ctypes.c_int32), ("n_layer", ctypes.c_int32),
                ("bos_token", ctypes.c_int32), ("temperature", ctypes.c_float),
                ("sparse_threshold", ctypes.c_float)]


class OrSqParams(ctypes.Structure):
    """SpectralQuantKVCacheConfig fields (src/spectralquant/types.rs:97-126)."""
    _fields_ = [("seed", ctypes.c_uint64), ("lloyd_max_iter", ctypes.c_int32),
                ("calibration_samples", ctypes.c_int32), ("avg_bits", ctypes.c_float),
                ("min_tail_bits", ctypes.c_int32), ("max_bits", ctypes.c_int32),
                ("wf_min_bits", ctypes.c_int32), ("wf_max_bits", ctypes.c_int32),
                ("use_water_fill", ctypes.c_int32)]


def sq_params(avg_bits=3.0, min_tail_bits=1, max_bits=8, lloyd_max_iter=30, calibration_samples=100, seed=42,
              use_water_fill=False, wf_min_bits=1, wf_max_bits=6):
    """The reference's test configuration (spectral_kv_cache.rs:1214-1234) by default."""
    return OrSqParams(seed, lloyd_max_iter, calibration_samples, avg_bits, min_tail_bits, max_bits, wf_min_bits,
                      wf_max_bits, int(use_water_fill))


SQ_LEVELS = 64


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIBPATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIBPATH):
            build()
        L = ctypes.CDLL(LIBPATH)
        P, I32, I64, F32, U64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_uint64
        cp = ctypes.POINTER(OrConfig)
        sig = {
            "or_rng_uniforms": (None, [U64, I64, P]),
            "or_rng_normals": (None, [U64, I64, P]),
            "or_rng_normals_rawstate": (None, [U64, I64, P]),
            "or_weights_count": (I64, [cp]),
            "or_weights_init": (None, [cp, U64, ctypes.c_int, F32, P]),
            "or_dot": (F32, [P, P, I64]),
            "or_sum_sq": (F32, [P, I64]),
            "or_sum": (F32, [P, I64]),
            "or_max": (F32, [P, I64]),
            "or_exp_inplace": (None, [P, I64]),
            "or_exp_sum_inplace": (F32, [P, I64]),
            "or_sparse_dot": (F32, [P, P, P, I64]),
            "or_softmax_scaled": (None, [P, I64, F32]),
            "or_sample_token": (I64, [P, I64, U64]),
            "or_sample_tokens": (None, [P, I64, I64, U64, P]),
            "or_verify_path": (I32, [P, P, P, I32, I64, U64, P]),
            "or_scalar_exp": (F32, [F32]),
            "or_tq_packed_len": (I64, [I64, ctypes.c_int]),
            "or_tq_codebook": (None, [I64, ctypes.c_int, P, P, P]),
            "or_tq_rotation": (None, [I64, U64, P]),
            "or_tq_rotation_from": (None, [I64, P, P]),
            "or_tq_store": (None, [P, P, ctypes.c_int, I64, P, P, P]),
            "or_tq_dequant": (None, [P, P, ctypes.c_int, I64, P, F32, P]),
            "or_tq_dequant_scalar": (None, [P, P, ctypes.c_int, I64, P, F32, P]),
            "or_tq_pack": (None, [P, I64, ctypes.c_int, P]),
            "or_tq_unpack": (None, [P, I64, ctypes.c_int, P]),
            "or_cosine": (F32, [P, P, I64]),
            "or_run_sequence": (ctypes.c_int, [cp, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, I32, P, P, P, P]),
            "or_run_batch": (ctypes.c_int, [cp, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, I32, I32, P, ctypes.c_int]),
            "or_run_sequence_rot": (ctypes.c_int, [cp, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, I32, P, P, P, P]),
            "or_prefill_then_decode": (ctypes.c_int, [cp, P, P, I32, P, I32, P]),
            "or_run_sequence_forced": (ctypes.c_int, [cp, ctypes.c_int, ctypes.c_int, P, P, I32, P, P]),
            "or_run_batch_tail": (ctypes.c_int, [cp, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, I32, I32, I32, P, ctypes.c_int]),
            "or_forward_paged": (ctypes.c_int, [cp, P, P, P, I64, I32, I32, P]),
            "or_sq_calibrate_eigenbasis": (ctypes.c_int, [P, I64, I64, P, P, P]),
            "or_sq_jacobi": (ctypes.c_int, [P, I64, P, P]),
            "or_spkv_predict": (None, [I64, I64, I64, F32, P, P]),
            "or_spkv_predictor_weights": (None, [I64, I64, I64, F32, P]),
            "or_set_lora": (ctypes.c_int, [ctypes.c_int, I64, I64, I64, F32, P, P]),
            "or_lora_apply": (None, [I64, I64, I64, F32, P, P, P, P]),
            "or_attention_head_gated": (None, [P, P, P, P, P, I64, I64, I64, I64, I64, F32, P]),
            "or_sq_quality_keys": (ctypes.c_int, [ctypes.POINTER(OrSqParams), I64, P, I64, I64, P]),
            "or_sq_allocate": (None, [F32, F32, I64, ctypes.c_int, P, P]),
            "or_sq_waterfill": (None, [P, I64, I64, ctypes.c_int, ctypes.c_int, P]),
            "or_sq_lloyd_fit": (None, [P, I64, ctypes.c_int, ctypes.c_int, U64, P]),
            "or_sq_nearest": (I64, [F32, P, I64]),
            "or_sq_pack": (I64, [P, P, I64, P]),
            "or_sq_unpack": (None, [P, I64, P, I64, P]),
            "or_sq_build": (ctypes.c_int, [ctypes.POINTER(OrSqParams), I64, I32, P, P, P, P, P, P, P, P]),
            "or_sq_roundtrip": (I64, [I64, P, P, P, P, P, P, P, P]),
            "or_run_sequence_sq": (ctypes.c_int, [cp, P, P, P, P, P, P, I32, P, P, P]),
            "or_time_decode": (ctypes.c_double, [cp, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, I32, I32, ctypes.c_int]),
        }
        for k, (r, a) in sig.items():
            f = getattr(L, k)
            f.restype = r
            f.argtypes = a
        _lib = L
    return _lib


def _p(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def config(vocab_size=27, block_size=16, n_embd=16, n_head=4, head_dim=4, n_kv_head=4,
           mlp_hidden=64, n_layer=1, bos_token=26, temperature=0.5, sparse_threshold=0.8):
    """Config::micro() by default (crates/katgpt-types/src/config.rs:226-316)."""
    return OrConfig(vocab_size, block_size, n_embd, n_head, head_dim, n_kv_head, mlp_hidden,
                    n_layer, bos_token, temperature, sparse_threshold)


def from_kg(kc):
    """OrConfig from a kgcuda.KgConfig."""
    return config(kc.vocab_size, kc.block_size, kc.n_embd, kc.n_head, kc.head_dim, kc.n_kv_head,
                  kc.mlp_hidden, kc.n_layer, kc.bos_token, kc.temperature, kc.sparse_threshold)


def normals(seed, n):
    out = np.empty(n, np.float32)
    lib().or_rng_normals(seed, n, _p(out))
    return out


def uniforms(seed, n):
    out = np.empty(n, np.float32)
    lib().or_rng_uniforms(seed, n, _p(out))
    return out


def weights(cfg, seed=42, scale_mode=0, std=0.02):
    n = lib().or_weights_count(ctypes.byref(cfg))
    w = np.empty(n, np.float32)
    lib().or_weights_init(ctypes.byref(cfg), seed, scale_mode, std, _p(w))
    return w


def dot(a, b):
    a, b = f32(a), f32(b)
    return lib().or_dot(_p(a), _p(b), a.size)


def sum_sq(x):
    x = f32(x)
    return lib().or_sum_sq(_p(x), x.size)


def vsum(x):
    x = f32(x)
    return lib().or_sum(_p(x), x.size)


def vmax(x):
    x = f32(x)
    return lib().or_max(_p(x), x.size)


def exp_inplace(x):
    x = f32(x).copy()
    lib().or_exp_inplace(_p(x), x.size)
    return x


def exp_sum_inplace(x):
    x = f32(x).copy()
    s = lib().or_exp_sum_inplace(_p(x), x.size)
    return x, s


def scalar_exp(v):
    return lib().or_scalar_exp(float(v))


def sparse_dot(w_row, idx, val):
    w_row, val = f32(w_row), f32(val)
    idx = np.ascontiguousarray(idx, dtype=np.int64)
    return lib().or_sparse_dot(_p(w_row), _p(idx), _p(val), idx.size)


def softmax_scaled(x, inv_temp):
    x = f32(x).copy()
    lib().or_softmax_scaled(_p(x), x.size, inv_temp)
    return x


def sample_token(probs, seed):
    p = f32(probs)
    return lib().or_sample_token(_p(p), p.size, seed)


def sample_tokens(probs, seed):
    """Successive draws of one Rng::new(seed): one token per row of probs [k][n]."""
    p = f32(probs)
    out = np.empty(p.shape[0], np.int64)
    lib().or_sample_tokens(_p(p), p.shape[1], p.shape[0], seed, _p(out))
    return out


def verify_path(p, q, drafts, seed):
    """The speculative acceptance loop for one path: (tokens, count)."""
    p, q = f32(p), f32(q)
    drafts = np.ascontiguousarray(drafts, np.int32)
    k = drafts.size
    out = np.zeros(k + 1, np.int32)
    cnt = lib().or_verify_path(_p(p), _p(q), _p(drafts), k, p.shape[-1], seed, _p(out))
    return out[:cnt], cnt


def packed_len(dim, bits):
    return lib().or_tq_packed_len(dim, bits)


def codebook(dim, bits):
    c = np.empty(1 << bits, np.float32)
    b = np.empty((1 << bits) - 1, np.float32)
    mse = ctypes.c_float()
    lib().or_tq_codebook(dim, bits, _p(c), _p(b), ctypes.byref(mse))
    return c, b, mse.value


def rotation(dim, seed=42):
    r = np.empty(dim * dim, np.float32)
    lib().or_tq_rotation(dim, seed, _p(r))
    return r.reshape(dim, dim)


def rotation_from(gauss):
    g = f32(gauss)
    dim = g.shape[0]
    r = np.empty(dim * dim, np.float32)
    lib().or_tq_rotation_from(dim, _p(g), _p(r))
    return r.reshape(dim, dim)


def normals_rawstate(state, n):
    out = np.empty(n, np.float32)
    lib().or_rng_normals_rawstate(state, n, _p(out))
    return out


def tq_store(rot, bnd, bits, x, packed_init=None):
    rot, bnd, x = f32(rot), f32(bnd), f32(x)
    dim = x.size
    pk = np.zeros(packed_len(dim, bits), np.uint8) if packed_init is None else np.array(packed_init, np.uint8)
    nrm = ctypes.c_float()
    lib().or_tq_store(_p(rot), _p(bnd), bits, dim, _p(x), _p(pk), ctypes.byref(nrm))
    return pk, nrm.value


def tq_dequant(rot_t, cent, bits, packed, norm):
    rot_t, cent = f32(rot_t), f32(cent)
    packed = np.ascontiguousarray(packed, np.uint8)
    dim = rot_t.shape[0]
    out = np.empty(dim, np.float32)
    lib().or_tq_dequant(_p(rot_t), _p(cent), bits, dim, _p(packed), norm, _p(out))
    return out


def tq_dequant_scalar(rot, cent, bits, packed, norm):
    rot, cent = f32(rot), f32(cent)
    packed = np.ascontiguousarray(packed, np.uint8)
    dim = rot.shape[0]
    out = np.empty(dim, np.float32)
    lib().or_tq_dequant_scalar(_p(rot), _p(cent), bits, dim, _p(packed), norm, _p(out))
    return out


def tq_pack(idx, bits):
    idx = np.ascontiguousarray(idx, np.uint8)
    out = np.zeros(packed_len(idx.size, bits), np.uint8)
    lib().or_tq_pack(_p(idx), idx.size, bits, _p(out))
    return out


def tq_unpack(packed, n, bits):
    packed = np.ascontiguousarray(packed, np.uint8)
    out = np.zeros(n, np.uint8)
    lib().or_tq_unpack(_p(packed), n, bits, _p(out))
    return out


def cosine(a, b):
    a, b = f32(a), f32(b)
    return lib().or_cosine(_p(a), _p(b), a.size)


def run_sequence(cfg, mode, w, tokens, key_bits=3, val_bits=3):
    """Teacher-forced forward of one sequence. Returns (logits[T,V], codes, norms, utilities)."""
    tokens = np.ascontiguousarray(tokens, np.int32)
    T = tokens.size
    logits = np.empty((T, cfg.vocab_size), np.float32)
    codes = norms = util = None
    if mode != MODE_BASE:
        kvd = cfg.n_kv_head * cfg.head_dim
        pl = packed_len(kvd, key_bits) + packed_len(kvd, val_bits)
        codes = np.zeros((cfg.n_layer, T, pl), np.uint8)
        norms = np.zeros((cfg.n_layer, T, 2), np.float32)
        util = np.zeros((cfg.n_layer, T), np.float32)
    rc = lib().or_run_sequence(ctypes.byref(cfg), mode, key_bits, val_bits, _p(f32(w)), _p(tokens), T,
                               _p(logits), _p(codes), _p(norms), _p(util))
    if rc:
        raise RuntimeError(f"or_run_sequence failed: {rc}")
    return logits, codes, norms, util


def run_sequence_rot(cfg, mode, w, tokens, key_bits=3, val_bits=3):
    """run_sequence for the quantized modes plus the rotated unit coordinates of
    every stored K/V vector: (logits[T,V], codes, norms, rot[L,T,2,kvd])."""
    tokens = np.ascontiguousarray(tokens, np.int32)
    T = tokens.size
    kvd = cfg.n_kv_head * cfg.head_dim
    logits = np.empty((T, cfg.vocab_size), np.float32)
    pl = packed_len(kvd, key_bits) + packed_len(kvd, val_bits)
    codes = np.zeros((cfg.n_layer, T, pl), np.uint8)
    norms = np.zeros((cfg.n_layer, T, 2), np.float32)
    rot = np.zeros((cfg.n_layer, T, 2, kvd), np.float32)
    rc = lib().or_run_sequence_rot(ctypes.byref(cfg), mode, key_bits, val_bits, _p(f32(w)), _p(tokens), T,
                                   _p(logits), _p(codes), _p(norms), _p(rot))
    if rc:
        raise RuntimeError(f"or_run_sequence_rot failed: {rc}")
    return logits, codes, norms, rot


def run_sequence_forced(cfg, w, tokens, codes, key_bits=3, val_bits=3):
    """forward_quantized of one sequence with every store's codes taken from
    codes[L][T][kpl + vpl] (norms computed as usual): logits [T][V]."""
    tokens = np.ascontiguousarray(tokens, np.int32)
    T = tokens.size
    kvd = cfg.n_kv_head * cfg.head_dim
    pl = packed_len(kvd, key_bits) + packed_len(kvd, val_bits)
    codes = np.ascontiguousarray(codes, np.uint8)
    if codes.shape != (cfg.n_layer, T, pl):
        raise ValueError(f"codes shape {codes.shape}, expected {(cfg.n_layer, T, pl)}")
    logits = np.empty((T, cfg.vocab_size), np.float32)
    rc = lib().or_run_sequence_forced(ctypes.byref(cfg), key_bits, val_bits, _p(f32(w)), _p(tokens), T, _p(codes),
                                      _p(logits))
    if rc:
        raise RuntimeError(f"or_run_sequence_forced failed: {rc}")
    return logits


def prefill_then_decode(cfg, w, prompt, cont=()):
    """forward_prefill of the prompt then forward_base of the continuation:
    logits [1 + len(cont)][V] (the prefill's last position first)."""
    prompt = np.ascontiguousarray(prompt, np.int32)
    cont = np.ascontiguousarray(cont, np.int32)
    out = np.empty((1 + cont.size, cfg.vocab_size), np.float32)
    rc = lib().or_prefill_then_decode(ctypes.byref(cfg), _p(f32(w)), _p(prompt), prompt.size,
                                      _p(cont) if cont.size else None, cont.size, _p(out))
    if rc:
        raise RuntimeError(f"or_prefill_then_decode failed: {rc}")
    return out


def run_batch(cfg, mode, w, tokens, key_bits=3, val_bits=3, threads=None, keep_logits=True, t0=0):
    tokens = np.ascontiguousarray(tokens, np.int32)
    n_seq, T = tokens.shape
    threads = threads or os.cpu_count() or 1
    logits = np.empty((n_seq, T - t0, cfg.vocab_size), np.float32) if keep_logits else None
    rc = lib().or_run_batch_tail(ctypes.byref(cfg), mode, key_bits, val_bits, _p(f32(w)), _p(tokens),
                                 n_seq, T, t0, _p(logits), threads)
    if rc:
        raise RuntimeError(f"or_run_batch failed: {rc}")
    return logits


def time_decode(cfg, w_one_layer, ctx, n_pos, mode=MODE_QUANT, key_bits=4, val_bits=4, threads=None):
    """tokens/s of forward_quantized (MODE_QUANT) or forward_base (MODE_BASE)
    decode at positions ctx.. (CPU-baseline timing; w_one_layer is the flat
    weights of the model with n_layer = 1, shared by every layer)."""
    threads = threads or os.cpu_count() or 1
    v = lib().or_time_decode(ctypes.byref(cfg), mode, key_bits, val_bits, _p(f32(w_one_layer)), ctx, n_pos,
                             threads)
    if v < 0:
        raise RuntimeError("or_time_decode: bad arguments")
    return v


PAGE_SIZE = 16  # crates/katgpt-transformer/src/kv_cache.rs:189


class PagedKVCache:
    """PagedKVCache (crates/katgpt-transformer/src/kv_cache.rs:187-420),
    restated: a pool of pages [K: PAGE_SIZE x kvd | V: PAGE_SIZE x kvd] f32,
    per-layer page tables per sequence, a LIFO free list and per-page
    reference counts. Integer bookkeeping only; the page data is a numpy
    array that grows like the reference's Vec<Vec<f32>>."""

    def __init__(self, cfg, max_sequences):  # :215-238
        self.kv_dim = cfg.n_kv_head * cfg.head_dim
        self.n_layer = cfg.n_layer
        initial = (cfg.block_size // PAGE_SIZE + 1) * cfg.n_layer
        self.pages = np.zeros((initial, 2, PAGE_SIZE, self.kv_dim), np.float32)
        self.layer_page_tables = [[[] for _ in range(max_sequences)] for _ in range(cfg.n_layer)]
        self.free_pages = list(range(initial))
        self.page_ref_counts = [0] * initial
        self.total_pages = initial

    def _alloc_page(self):  # :241-262
        if self.free_pages:
            idx = self.free_pages.pop()
            self.pages[idx] = 0.0
        else:
            self.pages = np.concatenate([self.pages, np.zeros((1, 2, PAGE_SIZE, self.kv_dim), np.float32)])
            idx = self.total_pages
            self.total_pages += 1
            self.page_ref_counts.append(0)
        self.page_ref_counts[idx] += 1
        return idx

    def ensure_pages(self, seq, pos):  # :268-296
        need = pos // PAGE_SIZE + 1
        for tables in self.layer_page_tables:
            while seq >= len(tables):
                tables.append([])
        deficits = [max(0, need - len(t[seq])) for t in self.layer_page_tables]
        new = [[self._alloc_page() for _ in range(df)] for df in deficits]
        for tables, pages in zip(self.layer_page_tables, new):
            tables[seq].extend(pages)

    def write_kv(self, layer, seq, pos, k, v):  # :298-309
        pg = self.layer_page_tables[layer][seq][pos // PAGE_SIZE]
        self.pages[pg, 0, pos % PAGE_SIZE] = k
        self.pages[pg, 1, pos % PAGE_SIZE] = v

    def read_kv(self, layer, seq, pos):  # :312-329
        pg = self.layer_page_tables[layer][seq][pos // PAGE_SIZE]
        return self.pages[pg, 0, pos % PAGE_SIZE].copy(), self.pages[pg, 1, pos % PAGE_SIZE].copy()

    def fork(self, seq, fork_at_pos):  # :334-350
        fork_page = fork_at_pos // PAGE_SIZE
        new_seq = len(self.layer_page_tables[0])
        for tables in self.layer_page_tables:
            shared = tables[seq][:min(fork_page, len(tables[seq]))]
            for pg in shared:
                self.page_ref_counts[pg] += 1
            tables.append(list(shared))
        return new_seq

    def rollback(self, seq, pos):  # :360-378
        keep = pos // PAGE_SIZE
        for tables in self.layer_page_tables:
            if seq >= len(tables):
                continue
            removed = tables[seq][keep:]
            del tables[seq][keep:]
            for pg in removed:
                self.page_ref_counts[pg] -= 1
                if self.page_ref_counts[pg] == 0:
                    self.free_pages.append(pg)

    def reset(self):  # :381-390
        for tables in self.layer_page_tables:
            for t in tables:
                self.free_pages.extend(t)
                t.clear()
        self.page_ref_counts = [0] * len(self.page_ref_counts)

    def table(self, seq, maxp):
        """The sequence's page lists as an int64 [n_layer][maxp] array (-1 past the end)."""
        out = np.full((self.n_layer, maxp), -1, np.int64)
        for l, tables in enumerate(self.layer_page_tables):
            t = tables[seq] if seq < len(tables) else []
            out[l, :len(t)] = t
        return out


def forward_paged(cfg, w, cache, seq, token, pos):
    """transformer::forward_paged (src/transformer.rs:3305-3504) of one token:
    ensure_pages, then the forward over `cache`'s pages; returns the logits."""
    cache.ensure_pages(seq, pos)
    maxp = max(len(t[seq]) for t in cache.layer_page_tables)
    tab = cache.table(seq, maxp)
    logits = np.empty(cfg.vocab_size, np.float32)
    rc = lib().or_forward_paged(ctypes.byref(cfg), _p(f32(w)), _p(cache.pages), _p(tab), maxp, token, pos,
                                _p(logits))
    if rc:
        raise RuntimeError(f"or_forward_paged failed: {rc}")
    return logits


def sq_calibrate_eigenbasis(samples):
    """calibrate_eigenbasis (src/spectralquant/spectral.rs:226-278) of samples [n][dim]:
    (eigenvectors [dim*dim] row-major, eigenvalues [dim], d_eff)."""
    x = f32(samples)
    n, dim = x.shape
    vec = np.empty(dim * dim, np.float32)
    val = np.empty(dim, np.float32)
    de = ctypes.c_float(0)
    rc = lib().or_sq_calibrate_eigenbasis(_p(x), n, dim, _p(vec), _p(val), ctypes.byref(de))
    if rc:
        raise RuntimeError(f"or_sq_calibrate_eigenbasis failed: {rc}")
    return vec, val, de.value


def sq_build(params, kvd, eig, evals, d_eff):
    """SpectralQuantKVCache::from_calibration tables for L layers (inputs [L][...]):
    dict of eig [L][kvd*kvd], bits [L][kvd] u8, cent [L][kvd][64], nlev [L][kvd], d_eff [L]."""
    eig = f32(eig).reshape(-1, kvd * kvd)
    L = eig.shape[0]
    evals = f32(evals).reshape(L, kvd)
    d_eff = f32(d_eff).reshape(L)
    out = dict(eig=np.empty((L, kvd * kvd), np.float32), bits=np.empty((L, kvd), np.uint8),
               cent=np.empty((L, kvd, SQ_LEVELS), np.float32), nlev=np.empty((L, kvd), np.int32),
               d_eff=np.empty(L, np.int32))
    rc = lib().or_sq_build(ctypes.byref(params), kvd, L, _p(eig), _p(evals), _p(d_eff), _p(out["eig"]),
                           _p(out["bits"]), _p(out["cent"]), _p(out["nlev"]), _p(out["d_eff"]))
    if rc:
        raise RuntimeError(f"or_sq_build failed: {rc}")
    return out


def sq_roundtrip(tabs, layer, x):
    """store_vector + dequantize_*_into of x with one layer's tables: (packed bytes, norm, dequantized)."""
    kvd = tabs["bits"].shape[1]
    x = f32(x)
    packed = np.zeros(kvd, np.uint8)
    norm = ctypes.c_float(0)
    deq = np.empty(kvd, np.float32)
    nb = lib().or_sq_roundtrip(kvd, _p(tabs["eig"][layer]), _p(tabs["bits"][layer]), _p(tabs["cent"][layer]),
                               _p(tabs["nlev"][layer]), _p(x), _p(packed), ctypes.byref(norm), _p(deq))
    if nb < 0:
        raise RuntimeError("or_sq_roundtrip: bad tables")
    return packed[:nb], norm.value, deq


def run_sequence_sq(cfg, w, tabs, tokens):
    """forward_quantized over SpectralQuantKVCache: (logits [T][V], codes [L][T][2*kvd], norms [L][T][2])."""
    tokens = np.ascontiguousarray(tokens, np.int32)
    T = tokens.size
    kvd = cfg.n_kv_head * cfg.head_dim
    logits = np.empty((T, cfg.vocab_size), np.float32)
    codes = np.zeros((cfg.n_layer, T, 2 * kvd), np.uint8)
    norms = np.zeros((cfg.n_layer, T, 2), np.float32)
    rc = lib().or_run_sequence_sq(ctypes.byref(cfg), _p(f32(w)), _p(tabs["eig"]), _p(tabs["bits"]),
                                  _p(tabs["cent"]), _p(tabs["nlev"]), _p(tokens), T, _p(logits), _p(codes),
                                  _p(norms))
    if rc:
        raise RuntimeError(f"or_run_sequence_sq failed: {rc}")
    return logits, codes, norms


def sq_jacobi(m):
    """jacobi_eigendecompose (spectral.rs:73-158) of a symmetric f64 matrix: (eigenvalues, eigenvectors row-major)."""
    m = np.ascontiguousarray(m, np.float64)
    d = m.shape[0]
    ev, vec = np.empty(d, np.float32), np.empty(d * d, np.float32)
    lib().or_sq_jacobi(_p(m), d, _p(ev), _p(vec))
    return ev, vec.reshape(d, d)


def sq_allocate(d_eff, avg_bits, head_dim, max_bits=8):
    """BitAllocator::allocate: (b_high, b_low)."""
    bh, bl = ctypes.c_int32(0), ctypes.c_int32(0)
    lib().or_sq_allocate(d_eff, avg_bits, head_dim, max_bits, ctypes.byref(bh), ctypes.byref(bl))
    return bh.value, bl.value


def sq_waterfill(ev, total, min_bits, max_bits=None):
    ev = np.ascontiguousarray(ev, np.float64)
    out = np.empty(ev.size, np.uint8)
    lib().or_sq_waterfill(_p(ev), ev.size, total, min_bits, -1 if max_bits is None else max_bits, _p(out))
    return out


def sq_lloyd_fit(data, bits, max_iter, seed):
    data = f32(data)
    out = np.empty(1 << bits, np.float32)
    lib().or_sq_lloyd_fit(_p(data) if data.size else None, data.size, bits, max_iter, seed, _p(out))
    return out


def sq_nearest(x, centroids):
    c = f32(centroids)
    return int(lib().or_sq_nearest(np.float32(x), _p(c), c.size))


def sq_pack(idx, bits):
    idx = np.ascontiguousarray(idx, np.uint8)
    bits = np.ascontiguousarray(bits, np.uint8)
    out = np.zeros(idx.size, np.uint8)
    n = lib().or_sq_pack(_p(idx), _p(bits), idx.size, _p(out))
    return out[:n]


def sq_unpack(packed, bits, n):
    packed = np.ascontiguousarray(packed, np.uint8)
    bits = np.ascontiguousarray(bits, np.uint8)
    out = np.empty(n, np.uint8)
    lib().or_sq_unpack(_p(packed), packed.size, _p(bits), n, _p(out))
    return out


def sq_quality_keys(params, keys, n_calib):
    """from_keys on keys[:n_calib], then store + dequantize of every key: reconstructions."""
    keys = f32(keys)
    out = np.empty_like(keys)
    rc = lib().or_sq_quality_keys(ctypes.byref(params), keys.shape[1], _p(keys), keys.shape[0], n_calib, _p(out))
    if rc:
        raise RuntimeError(f"or_sq_quality_keys failed: {rc}")
    return out


def spkv_predict(d_model, hidden, nkv, init_bias, h):
    """The SP-KV utility predictor (utility_predictor.rs:51-87) with its seeded weights: utilities [nkv]."""
    h = f32(h)
    out = np.empty(nkv, np.float32)
    lib().or_spkv_predict(d_model, hidden, nkv, init_bias, _p(h), _p(out))
    return out


def attention_head_gated(q, K, V, kvd, hd, tn, scale, bias=None, qoff=0, kvoff=0):
    """attention_head_gated (sp_kv/forward.rs:166-245): (out [len(q)], scores [tn])."""
    q, K, V = f32(q), f32(K), f32(V)
    out = np.zeros(q.size, np.float32)
    scores = np.zeros(tn, np.float32)
    b = None if bias is None else f32(bias)
    lib().or_attention_head_gated(_p(q), _p(K), _p(V), _p(out), _p(scores), qoff, kvoff, kvd, hd, tn, scale, _p(b))
    return out, scores


def lora_apply(a, b, alpha, x, out):
    """lora_apply (crates/katgpt-types/src/lora.rs:452-467): out + (alpha/rank) * B @ (A @ x)."""
    a, b, x = f32(a), f32(b), f32(x)
    out = f32(out).copy()
    rank, in_dim = a.shape
    lib().or_lora_apply(rank, in_dim, b.shape[0], alpha, _p(a), _p(b), _p(x), _p(out))
    return out


class lora_pair:
    """LoraPair (lora.rs:470-490) for the oracle's forwards while the block
    runs: `reader` = (A, B, alpha) for forward_prefill, `writer` for
    forward_base; None = no adapter."""

    def __init__(self, reader=None, writer=None):
        self.pair = (reader, writer)

    def __enter__(self):
        for which, ad in enumerate(self.pair):
            if ad is not None:
                a, b, alpha = f32(ad[0]), f32(ad[1]), float(ad[2])
                rc = lib().or_set_lora(which, a.shape[0], a.shape[1], b.shape[0], alpha, _p(a), _p(b))
                if rc:
                    raise ValueError("bad LoRA adapter")
        return self

    def __exit__(self, *exc):
        for which in (0, 1):
            lib().or_set_lora(which, 0, 0, 0, 0.0, None, None)
        return False
