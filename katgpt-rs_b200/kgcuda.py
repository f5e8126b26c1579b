"""ctypes host mirror of the reference `InferenceBackend` seam over libkgcuda.

`CudaBackend` follows the trait in src/inference_backend.rs:45-92 of
katgpt-rs (forward / device_name / supports_stateful / reset / compile /
is_compiled / recompile_hint) and adds the batched prefill/decode extension.
Every call goes through the C ABI declared in include/kg_abi.h; there is no
CPU fallback — if the shared library or a GPU is missing, construction fails.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBPATH = os.path.join(HERE, "lib", "libkgcuda.so")

KG_KV_F32, KG_KV_TQ, KG_KV_SPKV_TQ, KG_KV_PAGED, KG_KV_SQ = 0, 1, 2, 3, 4
KG_W_F32, KG_W_BF16 = 0, 1

STATUS = {0: "ok", -1: "invalid argument", -2: "device out of memory", -3: "CUDA error",
          -4: "timeout", -5: "weights not uploaded", -6: "unsupported configuration",
          -7: "invalid weights"}


class KgConfig(ctypes.Structure):
    """Mirror of kg_config (include/kg_abi.h)."""
    _fields_ = [
        ("vocab_size", ctypes.c_int32), ("block_size", ctypes.c_int32),
        ("n_embd", ctypes.c_int32), ("n_head", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("n_kv_head", ctypes.c_int32),
        ("mlp_hidden", ctypes.c_int32), ("n_layer", ctypes.c_int32),
        ("bos_token", ctypes.c_int32), ("temperature", ctypes.c_float),
        ("sparse_threshold", ctypes.c_float), ("kv_mode", ctypes.c_int32),
        ("key_bits", ctypes.c_int32), ("val_bits", ctypes.c_int32),
        ("weight_dtype", ctypes.c_int32), ("max_seqs", ctypes.c_int32),
        ("spkv_window", ctypes.c_int32), ("spkv_threshold", ctypes.c_float),
        ("spkv_init_bias", ctypes.c_float), ("tq_seed", ctypes.c_uint64),
    ]

    def kvd(self):
        return self.n_kv_head * self.head_dim


class KgSqParams(ctypes.Structure):
    """Mirror of kg_sq_params (SpectralQuantKVCacheConfig fields, include/kg_abi.h)."""
    _fields_ = [("seed", ctypes.c_uint64), ("lloyd_max_iter", ctypes.c_int32),
                ("calibration_samples", ctypes.c_int32), ("avg_bits", ctypes.c_float),
                ("min_tail_bits", ctypes.c_int32), ("max_bits", ctypes.c_int32),
                ("wf_min_bits", ctypes.c_int32), ("wf_max_bits", ctypes.c_int32),
                ("use_water_fill", ctypes.c_int32)]


SQ_LEVELS = 64


class KgError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status


_lib = None


def lib():
    """Load libkgcuda.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIBPATH):
            raise OSError(f"{LIBPATH} not built (run katgpt-rs_b200/build.py)")
        L = ctypes.CDLL(LIBPATH)
        P, I32, I64, F32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
        cfgp = ctypes.POINTER(KgConfig)
        sig = {
            "kg_config_micro": (None, [cfgp]),
            "kg_ctx_create": (ctypes.c_int, [cfgp, ctypes.c_int, ctypes.POINTER(P)]),
            "kg_ctx_destroy": (None, [P]),
            "kg_last_error": (ctypes.c_char_p, [P]),
            "kg_status_string": (ctypes.c_char_p, [ctypes.c_int]),
            "kg_device_name": (ctypes.c_char_p, [P]),
            "kg_weights_count": (I64, [cfgp]),
            "kg_reference_weights": (ctypes.c_int, [cfgp, ctypes.c_uint64, ctypes.c_int, F32, P]),
            "kg_upload_weights": (ctypes.c_int, [P, P, I64]),
            "kg_upload_weights_dev": (ctypes.c_int, [P, P, I64]),
            "kg_is_compiled": (ctypes.c_int, [P]),
            "kg_random_weights": (ctypes.c_int, [P, ctypes.c_uint64, F32]),
            "kg_download_weights": (ctypes.c_int, [P, P, I64]),
            "kg_seq_reset": (ctypes.c_int, [P, I32]),
            "kg_seq_reset_all": (ctypes.c_int, [P]),
            "kg_forward_token": (ctypes.c_int, [P, I32, I32, I32, P]),
            "kg_forward_batch": (ctypes.c_int, [P, I32, P, P, P, I32, P, P]),
            "kg_forward_batch_dev": (ctypes.c_int, [P, I32, P, P, P, I32, P, P, P]),
            "kg_tq_packed_len": (I64, [I64, I32]),
            "kg_tq_tables": (ctypes.c_int, [P, P, P, P, P, P]),
            "kg_tq_encode": (ctypes.c_int, [P, I32, I64, P, P, P]),
            "kg_tq_encode_noalloc": (ctypes.c_int, [P, I32, I64, P, P, P, P]),
            "kg_kv_codes": (ctypes.c_int, [P, I32, I32, I32, P, P, P]),
            "kg_spkv_utility": (ctypes.c_int, [P, I32, I32, I32, P]),
            "kg_profile": (ctypes.c_int, [P, ctypes.c_int]),
            "kg_profile_read": (ctypes.c_int, [P, P, P]),
            "kg_graph_kernels": (I64, [P]),
            "kg_seq_alloc": (ctypes.c_int, [P, P]),
            "kg_seq_free": (ctypes.c_int, [P, I32]),
            "kg_kv_snapshot_bytes": (I64, [P, I32]),
            "kg_kv_snapshot": (ctypes.c_int, [P, I32, I32, P, P]),
            "kg_kv_restore": (ctypes.c_int, [P, I32, I32, P, P]),
            "kg_set_mlp_hook": (ctypes.c_int, [P, F32, ctypes.c_uint64]),
            "kg_set_lora": (ctypes.c_int, [P, I32, I32, I32, I32, F32, P, P]),
            "kg_rng_seed": (ctypes.c_int, [P, I32, ctypes.c_uint64]),
            "kg_rng_state": (ctypes.c_int, [P, I32, P]),
            "kg_sample_dev": (ctypes.c_int, [P, I32, P, P, I64, P, P]),
            "kg_sample": (ctypes.c_int, [P, I32, P, P, P]),
            "kg_verify_dev": (ctypes.c_int, [P, I32, P, P, P, P, I32, P, P, P, P]),
            "kg_forward_prefill": (ctypes.c_int, [P, I32, P, P, I32, P]),
            "kg_forward_prefill_dev": (ctypes.c_int, [P, I32, P, P, I32, P, P]),
            "kg_verify": (ctypes.c_int, [P, I32, P, P, P, P, I32, P, P, P]),
            "kg_comm_unique_id": (ctypes.c_int, [P]),
            "kg_comm_init": (ctypes.c_int, [P, P, I32, I32]),
            "kg_comm_destroy": (ctypes.c_int, [P]),
            "kg_decode_gather_dev": (ctypes.c_int, [P, I32, P, P, P, P, P, P]),
            "kg_sq_params_default": (None, [ctypes.POINTER(KgSqParams)]),
            "kg_sq_calibrate": (ctypes.c_int, [P, ctypes.POINTER(KgSqParams), P, I64]),
            "kg_sq_calibrate_from": (ctypes.c_int, [P, ctypes.POINTER(KgSqParams), P, P, P]),
            "kg_sq_tables": (ctypes.c_int, [P, I32, P, P, P, P, P]),
            "kg_sq_calibrate_eigenbasis": (ctypes.c_int, [P, I64, I64, P, P, P]),
            "kg_sq_encode": (ctypes.c_int, [P, I32, I64, P, P, P]),
            "kg_sq_decode": (ctypes.c_int, [P, I32, I64, P, P, P]),
            "kg_sq_build_tables": (ctypes.c_int, [ctypes.POINTER(KgSqParams), I64, I32, P, P, P, P, P, P, P, P]),
            "kg_selftest_wait_timeout": (ctypes.c_int, [P, I64]),
            "kg_paged_init": (ctypes.c_int, [P, I32]),
            "kg_paged_ensure": (ctypes.c_int, [P, I32, I32]),
            "kg_paged_fork": (ctypes.c_int, [P, I32, I32, P]),
            "kg_paged_rollback": (ctypes.c_int, [P, I32, I32]),
            "kg_paged_reset": (ctypes.c_int, [P]),
            "kg_paged_write_kv": (ctypes.c_int, [P, I32, I32, I32, P, P]),
            "kg_paged_read_kv": (ctypes.c_int, [P, I32, I32, I32, P, P]),
            "kg_paged_table": (ctypes.c_int, [P, I32, I32, P, I32, P]),
            "kg_paged_stats": (ctypes.c_int, [P, P, P, P, P, I64]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def exported_symbols():
    """Names of every kg_* function the header declares (for ABI checks)."""
    lib()
    return sorted(n for n in dir(_lib) if n.startswith("kg_"))


def comm_unique_id():
    """A 128-byte NCCL unique id (bytes) for kg_comm_init."""
    buf = (ctypes.c_uint8 * 128)()
    rc = lib().kg_comm_unique_id(buf)
    if rc:
        raise KgError(rc, "kg_comm_unique_id")
    return bytes(buf)


def bf16_round(a):
    """Round f32 to bf16 (nearest-even) and back, as the device does on upload."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def micro_config(**kw):
    c = KgConfig()
    lib().kg_config_micro(ctypes.byref(c))
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def _ptr(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def reference_weights(cfg, seed=42, scale_mode=0, std=0.02):
    """TransformerWeights::new(config, Rng::new(seed)) in the flat layout."""
    n = lib().kg_weights_count(ctypes.byref(cfg))
    w = np.empty(n, np.float32)
    rc = lib().kg_reference_weights(ctypes.byref(cfg), seed, scale_mode, std, _ptr(w))
    if rc:
        raise KgError(rc, "kg_reference_weights")
    return w


class CudaBackend:
    """InferenceBackend for one B200, backed by libkgcuda (one context)."""

    def __init__(self, cfg, device=0):
        self.cfg = cfg
        self._h = ctypes.c_void_p()
        rc = lib().kg_ctx_create(ctypes.byref(cfg), device, ctypes.byref(self._h))
        if rc:
            raise KgError(rc, "kg_ctx_create")

    def close(self):
        if self._h:
            lib().kg_ctx_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc):
        if rc:
            raise KgError(rc, lib().kg_last_error(self._h).decode())

    # ---- trait methods
    def device_name(self):
        return lib().kg_device_name(self._h).decode()

    def supports_stateful(self):
        return True  # the KV cache lives on the device

    def compile(self, weights):
        w = np.ascontiguousarray(weights, dtype=np.float32)
        self._check(lib().kg_upload_weights(self._h, _ptr(w), w.size))

    def random_weights(self, seed=0, std=0.02):
        """Synthetic N(0, std) bf16 weights generated on the device (bf16 path)."""
        self._check(lib().kg_random_weights(self._h, seed, std))

    def download_weights(self):
        n = lib().kg_weights_count(ctypes.byref(self.cfg))
        w = np.empty(n, np.float32)
        self._check(lib().kg_download_weights(self._h, _ptr(w), n))
        return w

    def is_compiled(self):
        return bool(lib().kg_is_compiled(self._h))

    def recompile_hint(self):
        pass  # weights are re-uploaded explicitly with compile()

    def reset(self, seq=None):
        if seq is None:
            self._check(lib().kg_seq_reset_all(self._h))
        else:
            self._check(lib().kg_seq_reset(self._h, seq))

    def forward(self, token, pos, seq=0):
        out = np.empty(self.cfg.vocab_size, np.float32)
        self._check(lib().kg_forward_token(self._h, seq, token, pos, _ptr(out)))
        return out

    # ---- batched extension
    def forward_batch(self, tokens, seq_ids=None, start_pos=None, probs=False, logits=True):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        if tokens.ndim == 1:
            tokens = tokens[:, None]
        n_seq, T = tokens.shape
        ids = np.arange(n_seq, dtype=np.int32) if seq_ids is None else np.ascontiguousarray(seq_ids, np.int32)
        sp = None if start_pos is None else np.ascontiguousarray(start_pos, np.int32)
        V = self.cfg.vocab_size
        lo = np.empty((n_seq, T, V), np.float32) if logits else None
        pr = np.empty((n_seq, T, V), np.float32) if probs else None
        self._check(lib().kg_forward_batch(self._h, n_seq, _ptr(ids), _ptr(tokens), _ptr(sp), T,
                                           _ptr(lo), _ptr(pr)))
        if probs and logits:
            return lo, pr
        return lo if logits else pr

    def forward_prefill(self, tokens, seq_ids=None):
        """forward_prefill (bidirectional) over each row of tokens from position 0:
        the last position's logits [n_seq][vocab]."""
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        n_seq, T = tokens.shape
        ids = np.arange(n_seq, dtype=np.int32) if seq_ids is None else np.ascontiguousarray(seq_ids, np.int32)
        out = np.empty((n_seq, self.cfg.vocab_size), np.float32)
        self._check(lib().kg_forward_prefill(self._h, n_seq, _ptr(ids), _ptr(tokens), T, _ptr(out)))
        return out

    def forward_batch_dev(self, n_seq, T, ids_ptr, tok_ptr, pos_ptr, logits_ptr, probs_ptr, stream_ptr):
        """Device-pointer form (integers are raw device addresses)."""
        self._check(lib().kg_forward_batch_dev(self._h, n_seq, ids_ptr, tok_ptr, pos_ptr, T,
                                               logits_ptr, probs_ptr, stream_ptr))

    # ---- codec access
    def tq_tables(self):
        kvd = self.cfg.kvd()
        rot = np.empty(kvd * kvd, np.float32)
        nk, nv = 1 << self.cfg.key_bits, 1 << self.cfg.val_bits
        kc, kb = np.empty(nk, np.float32), np.empty(nk - 1, np.float32)
        vc, vb = np.empty(nv, np.float32), np.empty(nv - 1, np.float32)
        self._check(lib().kg_tq_tables(self._h, _ptr(rot), _ptr(kc), _ptr(kb), _ptr(vc), _ptr(vb)))
        return rot.reshape(kvd, kvd), kc, kb, vc, vb

    def tq_encode(self, x, which=0, packed_init=None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        n_vec = x.shape[0]
        bits = self.cfg.key_bits if which == 0 else self.cfg.val_bits
        pl = lib().kg_tq_packed_len(self.cfg.kvd(), bits)
        packed = np.zeros((n_vec, pl), np.uint8) if packed_init is None else np.array(packed_init, np.uint8)
        norms = np.empty(n_vec, np.float32)
        self._check(lib().kg_tq_encode(self._h, which, n_vec, _ptr(x), _ptr(packed), _ptr(norms)))
        return packed, norms

    def kv_codes(self, seq, layer, pos):
        kvd = self.cfg.kvd()
        sq = self.cfg.kv_mode == KG_KV_SQ  # SpectralQuant: kv_dim-byte rows, the pack in front
        kp = np.empty(kvd if sq else lib().kg_tq_packed_len(kvd, self.cfg.key_bits), np.uint8)
        vp = np.empty(kvd if sq else lib().kg_tq_packed_len(kvd, self.cfg.val_bits), np.uint8)
        nr = np.empty(2, np.float32)
        self._check(lib().kg_kv_codes(self._h, seq, layer, pos, _ptr(kp), _ptr(vp), _ptr(nr)))
        return kp, vp, nr

    def kv_codes_all(self, seq, T):
        """Every stored code of one sequence, positions 0..T-1: [n_layer][T][kpl + vpl] (K then V)."""
        rows = []
        for layer in range(self.cfg.n_layer):
            for pos in range(T):
                kp, vp, _ = self.kv_codes(seq, layer, pos)
                rows.append(np.concatenate([kp, vp]))
        return np.stack(rows).reshape(self.cfg.n_layer, T, -1)

    def profile(self, enable=True):
        self._check(lib().kg_profile(self._h, 1 if enable else 0))

    def profile_read(self):
        """Summed device ms and interval counts per phase (attn, encode, gemm)."""
        ms = np.zeros(3, np.float32)
        cnt = np.zeros(3, np.int64)
        self._check(lib().kg_profile_read(self._h, _ptr(ms), _ptr(cnt)))
        return ms, cnt

    def seq_alloc(self):
        """A free sequence slot (reset), as kg_seq_alloc."""
        out = ctypes.c_int32(-1)
        self._check(lib().kg_seq_alloc(self._h, ctypes.byref(out)))
        return out.value

    def seq_free(self, seq):
        self._check(lib().kg_seq_free(self._h, seq))

    def kv_snapshot_bytes(self, pos):
        return int(lib().kg_kv_snapshot_bytes(self._h, pos))

    def kv_snapshot(self, seq, pos, dst_dev, stream=None):
        """Copy positions [0, pos) of `seq` into device memory at dst_dev (int address)."""
        self._check(lib().kg_kv_snapshot(self._h, seq, pos, ctypes.c_void_p(dst_dev), stream))

    def kv_restore(self, seq, pos, src_dev, stream=None):
        self._check(lib().kg_kv_restore(self._h, seq, pos, ctypes.c_void_p(src_dev), stream))

    def set_lora(self, which, a=None, b=None, alpha=0.0):
        """LoraPair adapter (crates/katgpt-types/src/lora.rs): which 0 = reader
        (forward_prefill), 1 = writer (forward_batch / forward); A [rank][in_dim],
        B [out_dim][rank]; a None adapter removes it."""
        if a is None:
            self._check(lib().kg_set_lora(self._h, which, 0, 0, 0, 0.0, None, None))
            return
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        if a.ndim != 2 or b.ndim != 2 or b.shape[1] != a.shape[0]:
            raise ValueError("LoRA: A [rank][in_dim] and B [out_dim][rank]")
        self._check(lib().kg_set_lora(self._h, which, a.shape[0], a.shape[1], b.shape[0], float(alpha),
                                      _ptr(a), _ptr(b)))

    def set_mlp_hook(self, keep, seed=0):
        """Benchmark hook: Bernoulli(keep) sparse hidden activations after W1 (0 = off)."""
        self._check(lib().kg_set_mlp_hook(self._h, keep, seed))

    def graph_kernels(self):
        """Kernel launches replayed by the last forward call's CUDA graph (0: eager)."""
        return int(lib().kg_graph_kernels(self._h))

    # ---- sampling (sample_token_into on the device)
    def rng_seed(self, seq, seed):
        self._check(lib().kg_rng_seed(self._h, seq, seed))

    def rng_state(self, seq):
        out = ctypes.c_uint64(0)
        self._check(lib().kg_rng_state(self._h, seq, ctypes.byref(out)))
        return out.value

    def sample(self, probs, seq_ids=None):
        """Token ids drawn from probs [n_rows][vocab] with each row's slot generator."""
        probs = np.ascontiguousarray(probs, dtype=np.float32)
        n = probs.shape[0]
        ids = np.arange(n, dtype=np.int32) if seq_ids is None else np.ascontiguousarray(seq_ids, np.int32)
        out = np.empty(n, np.int32)
        self._check(lib().kg_sample(self._h, n, _ptr(ids), _ptr(probs), _ptr(out)))
        return out

    def verify(self, tokens, drafts, draft_probs, start_pos, seq_ids=None):
        """Speculative verification of one draft path per sequence (kg_verify):
        returns (accepted [n][k+1], n_accepted [n])."""
        drafts = np.ascontiguousarray(drafts, np.int32)
        n, k = drafts.shape
        tokens = np.ascontiguousarray(tokens, np.int32)
        start_pos = np.ascontiguousarray(start_pos, np.int32)
        q = np.ascontiguousarray(draft_probs, np.float32)
        ids = np.arange(n, dtype=np.int32) if seq_ids is None else np.ascontiguousarray(seq_ids, np.int32)
        acc = np.zeros((n, k + 1), np.int32)
        cnt = np.zeros(n, np.int32)
        self._check(lib().kg_verify(self._h, n, _ptr(ids), _ptr(start_pos), _ptr(tokens), _ptr(drafts), k, _ptr(q),
                                    _ptr(acc), _ptr(cnt)))
        return acc, cnt

    # ---- multi-GPU sequence shards
    def comm_init(self, uid, world, rank):
        """Join the NCCL communicator `uid` (bytes from comm_unique_id()) as `rank`."""
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(bytes(uid))
        self._check(lib().kg_comm_init(self._h, buf, world, rank))

    def comm_destroy(self):
        self._check(lib().kg_comm_destroy(self._h))

    def decode_gather_dev(self, n_seq, ids_ptr, tok_ptr, pos_ptr, logits_all_ptr, tokens_all_ptr, stream_ptr):
        """One decode step of this rank's sequences, then the all-gather (device pointers)."""
        self._check(lib().kg_decode_gather_dev(self._h, n_seq, ids_ptr, tok_ptr, pos_ptr, logits_all_ptr,
                                               tokens_all_ptr, stream_ptr))

    def spkv_utility(self, seq, layer, pos):
        u = np.empty(1, np.float32)
        self._check(lib().kg_spkv_utility(self._h, seq, layer, pos, _ptr(u)))
        return float(u[0])

    # ---- PagedKVCache (kv_mode KG_KV_PAGED; crates/katgpt-transformer/src/kv_cache.rs:187-420)

    def paged_init(self, max_sequences):
        """PagedKVCache::new(config, max_sequences)."""
        self._check(lib().kg_paged_init(self._h, max_sequences))

    def paged_ensure(self, seq, pos):
        self._check(lib().kg_paged_ensure(self._h, seq, pos))

    def paged_fork(self, seq, fork_at_pos):
        out = ctypes.c_int32(-1)
        self._check(lib().kg_paged_fork(self._h, seq, fork_at_pos, ctypes.byref(out)))
        return out.value

    def paged_rollback(self, seq, pos):
        self._check(lib().kg_paged_rollback(self._h, seq, pos))

    def paged_reset(self):
        self._check(lib().kg_paged_reset(self._h))

    def paged_write_kv(self, layer, seq, pos, k, v):
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        self._check(lib().kg_paged_write_kv(self._h, layer, seq, pos, _ptr(k), _ptr(v)))

    def paged_read_kv(self, layer, seq, pos):
        kvd = self.cfg.kvd()
        k = np.empty(kvd, np.float32)
        v = np.empty(kvd, np.float32)
        self._check(lib().kg_paged_read_kv(self._h, layer, seq, pos, _ptr(k), _ptr(v)))
        return k, v

    def paged_table(self, layer, seq):
        n = ctypes.c_int32(0)
        self._check(lib().kg_paged_table(self._h, layer, seq, None, 0, ctypes.byref(n)))
        out = np.empty(n.value, np.int32)
        self._check(lib().kg_paged_table(self._h, layer, seq, _ptr(out), n.value, ctypes.byref(n)))
        return [int(x) for x in out]

    def paged_stats(self):
        """(total_pages, free_pages, n_sequences, page_ref_counts)."""
        tot, free, ns = ctypes.c_int64(0), ctypes.c_int64(0), ctypes.c_int32(0)
        self._check(lib().kg_paged_stats(self._h, ctypes.byref(tot), ctypes.byref(free), ctypes.byref(ns), None, 0))
        refs = np.zeros(tot.value, np.int32)
        self._check(lib().kg_paged_stats(self._h, None, None, None, _ptr(refs), tot.value))
        return tot.value, free.value, ns.value, [int(r) for r in refs]

    # ---- SpectralQuant (kv_mode KG_KV_SQ; src/spectralquant/)

    def sq_calibrate(self, key_samples, params=None):
        """SpectralQuantKVCache::from_keys on key_samples [n][kv_dim]."""
        x = np.ascontiguousarray(key_samples, np.float32)
        p = params or sq_params()
        self._check(lib().kg_sq_calibrate(self._h, ctypes.byref(p), _ptr(x), x.shape[0]))

    def sq_calibrate_from(self, eigenvectors, eigenvalues, d_eff, params=None):
        """SpectralQuantKVCache::from_calibration: per layer [L][kvd*kvd], [L][kvd], [L]."""
        e = np.ascontiguousarray(eigenvectors, np.float32)
        v = np.ascontiguousarray(eigenvalues, np.float32)
        d = np.ascontiguousarray(d_eff, np.float32)
        p = params or sq_params()
        self._check(lib().kg_sq_calibrate_from(self._h, ctypes.byref(p), _ptr(e), _ptr(v), _ptr(d)))

    def sq_encode(self, x, layer=0, packed_init=None):
        """store_vector of x [n][kv_dim]: (packed [n][kv_dim], norms [n])."""
        x = np.ascontiguousarray(x, np.float32)
        n, kvd = x.shape
        packed = np.zeros((n, kvd), np.uint8) if packed_init is None else np.array(packed_init, np.uint8, copy=True)
        norms = np.empty(n, np.float32)
        self._check(lib().kg_sq_encode(self._h, layer, n, _ptr(x), _ptr(packed), _ptr(norms)))
        return packed, norms

    def sq_decode(self, packed, norms, layer=0):
        """dequantize_*_into of packed rows [n][kv_dim] with norms [n]: [n][kv_dim] f32."""
        packed = np.ascontiguousarray(packed, np.uint8)
        norms = np.ascontiguousarray(norms, np.float32)
        out = np.empty((packed.shape[0], self.cfg.kvd()), np.float32)
        self._check(lib().kg_sq_decode(self._h, layer, packed.shape[0], _ptr(packed), _ptr(norms), _ptr(out)))
        return out

    def sq_tables(self, layer):
        """(eigenvectors [kvd*kvd], bits [kvd], centroids [kvd][64], n_levels [kvd], d_eff) of one layer."""
        kvd = self.cfg.kvd()
        e = np.empty(kvd * kvd, np.float32)
        b = np.empty(kvd, np.uint8)
        c = np.empty((kvd, SQ_LEVELS), np.float32)
        n = np.empty(kvd, np.int32)
        d = ctypes.c_int32(0)
        self._check(lib().kg_sq_tables(self._h, layer, _ptr(e), _ptr(b), _ptr(c), _ptr(n), ctypes.byref(d)))
        return e, b, c, n, d.value


def sq_params(**kw):
    """kg_sq_params_default (the reference's test configuration) with overrides."""
    p = KgSqParams()
    lib().kg_sq_params_default(ctypes.byref(p))
    for k, v in kw.items():
        setattr(p, k, v)
    return p


def sq_calibrate_eigenbasis(samples):
    """kg_sq_calibrate_eigenbasis (host): (eigenvectors [dim*dim], eigenvalues [dim], d_eff)."""
    x = np.ascontiguousarray(samples, np.float32)
    n, dim = x.shape
    vec = np.empty(dim * dim, np.float32)
    val = np.empty(dim, np.float32)
    de = ctypes.c_float(0)
    rc = lib().kg_sq_calibrate_eigenbasis(_ptr(x), n, dim, _ptr(vec), _ptr(val), ctypes.byref(de))
    if rc:
        raise KgError(rc, "kg_sq_calibrate_eigenbasis")
    return vec, val, de.value


def sq_build_tables(params, kvd, eig, evals, d_eff):
    """kg_sq_build_tables (host): dict of eig, bits, cent, nlev, d_eff per layer."""
    eig = np.ascontiguousarray(eig, np.float32).reshape(-1, kvd * kvd)
    L = eig.shape[0]
    evals = np.ascontiguousarray(evals, np.float32).reshape(L, kvd)
    d_eff = np.ascontiguousarray(d_eff, np.float32).reshape(L)
    out = dict(eig=np.empty((L, kvd * kvd), np.float32), bits=np.empty((L, kvd), np.uint8),
               cent=np.empty((L, kvd, SQ_LEVELS), np.float32), nlev=np.empty((L, kvd), np.int32),
               d_eff=np.empty(L, np.int32))
    rc = lib().kg_sq_build_tables(ctypes.byref(params), kvd, L, _ptr(eig), _ptr(evals), _ptr(d_eff),
                                  _ptr(out["eig"]), _ptr(out["bits"]), _ptr(out["cent"]), _ptr(out["nlev"]),
                                  _ptr(out["d_eff"]))
    if rc:
        raise KgError(rc, "kg_sq_build_tables")
    return out


class DDTreeBranchCache:
    """DDTreeBranchCache (src/speculative/types.rs:218-290) over a context
    created with kv_mode KG_KV_PAGED: the trunk is sequence 0, forks share
    whole prefix pages, and the branch budget behaves as the reference's
    (a fork past max_branches returns the source sequence; discarding a
    branch other than the trunk frees its pages and its budget slot)."""

    def __init__(self, backend, max_branches):
        self.backend = backend
        self.max_branches = max_branches
        self.branch_count = 1  # sequence 0 = trunk
        backend.paged_init(max_branches)  # PagedKVCache::new(config, max_branches)

    def fork_branch(self, src, at_pos):
        if self.branch_count >= self.max_branches:
            return src  # budget exhausted: reuse the source
        new_seq = self.backend.paged_fork(src, at_pos)
        self.branch_count += 1
        return new_seq

    def forward_branch(self, seq_idx, token, pos):
        """forward_paged of one token of a branch: logits [vocab]."""
        return self.backend.forward(token, pos, seq=seq_idx)

    def rollback_branch(self, seq_idx, at_pos):
        self.backend.paged_rollback(seq_idx, at_pos)

    def discard_branch(self, seq_idx):
        self.backend.paged_rollback(seq_idx, 0)
        if seq_idx > 0 and self.branch_count > 1:
            self.branch_count -= 1

    def reset(self):
        self.backend.paged_reset()
        self.branch_count = 1
