"""ctypes binding of include/sana_cuda.h.

``SanaCuda`` wraps one handle. Its single-op methods have the names, argument meaning and
layouts of the CPU checkers in ``oracle/oracle.py`` (which follow the reference's
functions), so the same known-answer and parity cases run against either. Errors map to
``ValueError`` for SANA_ERR_INVALID (the reference's std::invalid_argument) and
``SanaError`` otherwise.
"""
from __future__ import annotations

import ctypes
import os
from typing import List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)

SANA_MODE_BF16, SANA_MODE_F32 = 0, 1
SANA_LAYOUT_REFERENCE, SANA_LAYOUT_TORCH = 0, 1
_ERRS = {1: "SANA_ERR_INVALID", 2: "SANA_ERR_CUDA", 3: "SANA_ERR_TIMEOUT", 4: "SANA_ERR_STATE", 5: "SANA_ERR_NOMEM"}

_f32p = ctypes.POINTER(ctypes.c_float)
_i = ctypes.c_int
_f = ctypes.c_float


class SanaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{_ERRS.get(code, code)}: {msg}")
        self.code = code


class sana_dims(ctypes.Structure):
    _fields_ = [("n_blocks", _i), ("hidden", _i), ("latent_channels", _i), ("caption_dim", _i),
                ("ff_expanded", _i), ("self_heads", _i), ("cross_heads", _i)]


def lib_path() -> str:
    return os.environ.get("SANA_CUDA_LIB", os.path.join(PKG, "lib", "libsana_cuda.so"))


_LIB = None


def load_library():
    """Loads the in-tree shared library (raises if it has not been built)."""
    global _LIB
    if _LIB is None:
        path = lib_path()
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is missing: run python sana.cpp_b200/build.py")
        lib = ctypes.CDLL(path)
        lib.sana_cuda_last_error.restype = ctypes.c_char_p
        lib.sana_cuda_last_error.argtypes = [ctypes.c_void_p]
        lib.sana_cuda_stream.restype = ctypes.c_void_p
        lib.sana_cuda_stream.argtypes = [ctypes.c_void_p]
        lib.sana_cuda_destroy.argtypes = [ctypes.c_void_p]
        lib.sana_cuda_last_launch_count.argtypes = [ctypes.c_void_p]
        if hasattr(lib, "sana_cuda_vae_last_launch_count"):
            lib.sana_cuda_vae_last_launch_count.argtypes = [ctypes.c_void_p]
        lib.sana_randn_torch_cpu.argtypes = [_f32p, ctypes.c_size_t, ctypes.c_uint64]
        lib.sana_gguf_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p,
                                       ctypes.c_size_t]
        lib.sana_gguf_close.argtypes = [ctypes.c_void_p]
        lib.sana_gguf_tensor_count.argtypes = [ctypes.c_void_p]
        lib.sana_gguf_find.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
        lib.sana_gguf_tensor_info.argtypes = [ctypes.c_void_p, _i, ctypes.POINTER(ctypes.c_char_p),
                                              ctypes.POINTER(_i), ctypes.POINTER(_i),
                                              ctypes.POINTER(ctypes.c_int64), _i, ctypes.POINTER(ctypes.c_void_p),
                                              ctypes.POINTER(ctypes.c_uint64)]
        _LIB = lib
    return _LIB


def _ptr(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_f32p)


def _f32(a) -> Optional[np.ndarray]:
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def randn_torch_cpu(n: int, seed: int) -> np.ndarray:
    """torch.randn(n) on a CPU generator seeded with `seed` (n >= 16), bit-identical to the
    reference's randn_torch_cpu."""
    out = np.empty(n, np.float32)
    rc = load_library().sana_randn_torch_cpu(_ptr(out), ctypes.c_size_t(n), ctypes.c_uint64(seed))
    if rc != 0:
        raise ValueError("randn_torch_cpu needs at least 16 elements")
    return out


GGUF_F32, GGUF_F16, GGUF_BF16 = 0, 1, 30


def gguf_index(path: str) -> dict:
    """The library's GGUF reader on one file: {name: (element type, shape, array)} with the
    shape slowest-first and, for fp32 / fp16 tensors, a copy of the data (None otherwise)."""
    lib = load_library()
    h = ctypes.c_void_p()
    err = ctypes.create_string_buffer(512)
    rc = lib.sana_gguf_open(os.fsencode(path), ctypes.byref(h), err, 512)
    if rc != 0:
        raise SanaError(rc, err.value.decode())
    try:
        out = {}
        for i in range(lib.sana_gguf_tensor_count(h)):
            name, typ, rank = ctypes.c_char_p(), _i(), _i()
            shape = (ctypes.c_int64 * 8)()
            data, nbytes = ctypes.c_void_p(), ctypes.c_uint64()
            lib.sana_gguf_tensor_info(h, _i(i), ctypes.byref(name), ctypes.byref(typ), ctypes.byref(rank), shape, 8,
                                      ctypes.byref(data), ctypes.byref(nbytes))
            shp = tuple(shape[d] for d in range(rank.value))
            arr = None
            dt = {GGUF_F32: np.float32, GGUF_F16: np.float16}.get(typ.value)
            if dt is not None and nbytes.value:
                buf = (ctypes.c_char * nbytes.value).from_address(data.value)
                arr = np.frombuffer(bytes(buf), dtype=dt).reshape(shp)
            out[name.value.decode()] = (typ.value, shp, arr)
        return out
    finally:
        lib.sana_gguf_close(h)


def _host_status(rc: int, err) -> None:
    if rc == 1:
        raise ValueError(err.value.decode())
    if rc != 0:
        raise SanaError(rc, err.value.decode())


def select_rows_first_and_last(x, keep: int) -> np.ndarray:
    """gemma_encoder.cpp:51-77 through the library: row 0 of x [rows, cols], then its last
    keep-1 rows."""
    x = _f32(x)
    if x.ndim != 2:
        raise ValueError("select_rows_first_and_last expects a rank-2 tensor")
    rows, cols = x.shape
    out = np.empty((max(int(keep), 0), cols), np.float32)
    err = ctypes.create_string_buffer(256)
    _host_status(load_library().sana_select_rows_first_and_last(
        _ptr(x), ctypes.c_size_t(rows), ctypes.c_size_t(cols), ctypes.c_size_t(max(int(keep), 0)),
        _ptr(out), err, 256), err)
    return out


def prompt_pair_assemble(negative, negative_real: int, positive, positive_real: int, max_sequence_length: int = 300):
    """The tail of encode_prompt_pair (gemma_encoder.cpp:188-244) through the library:
    (embeddings [2, L, hidden] negative first, bias [2, 1, L])."""
    negative, positive = _f32(negative), _f32(positive)
    L = int(max_sequence_length)
    hidden = positive.shape[1]
    if negative.ndim != 2 or positive.ndim != 2 or negative.shape[1] != hidden:
        raise ValueError("negative and positive hidden states must be [rows, hidden] with the same hidden size")
    emb = np.empty((2, L, hidden), np.float32)
    bias = np.empty((2, 1, L), np.float32)
    err = ctypes.create_string_buffer(256)
    _host_status(load_library().sana_prompt_pair_assemble(
        _ptr(negative), ctypes.c_size_t(negative.shape[0]), ctypes.c_size_t(negative_real), _ptr(positive),
        ctypes.c_size_t(positive.shape[0]), ctypes.c_size_t(positive_real), ctypes.c_size_t(hidden),
        ctypes.c_size_t(L), _ptr(emb), _ptr(bias), err, 256), err)
    return emb, bias


def gemm_counts():
    """(tensor-core GEMM launches, CUDA-core GEMM launches) in this process."""
    a, b = ctypes.c_longlong(0), ctypes.c_longlong(0)
    load_library().sana_cuda_gemm_counts(ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value


def scheduler_schedule(n: int, flow_shift: float = 3.0):
    ts = np.empty(n, np.float32)
    sg = np.empty(n + 1, np.float32)
    rc = load_library().sana_scheduler_schedule(_i(n), _f(flow_shift), _ptr(ts), _ptr(sg))
    if rc != 0:
        raise ValueError("num_inference_steps must be positive")
    return ts, sg


class sana_scheduler_config(ctypes.Structure):
    """SanaSchedulerConfig (scheduler.h:9-20) as the C ABI carries it."""
    _fields_ = [("num_train_timesteps", _i), ("flow_shift", _f), ("use_flow_sigmas", _i), ("solver_order", _i),
                ("lower_order_final", _i), ("final_sigmas_zero", _i), ("solver_heun", _i)]


SCHEDULER_DEFAULTS = dict(num_train_timesteps=1000, flow_shift=3.0, use_flow_sigmas=1, solver_order=2,
                          lower_order_final=1, final_sigmas_zero=1, solver_heun=0)


def scheduler_config(**kw) -> sana_scheduler_config:
    """A config with the reference's defaults (make_sana_scheduler_config) except `kw`."""
    bad = set(kw) - set(SCHEDULER_DEFAULTS)
    if bad:
        raise TypeError(f"unknown scheduler config fields {sorted(bad)}")
    return sana_scheduler_config(**{**SCHEDULER_DEFAULTS, **kw})


def scheduler_schedule_config(n: int, **kw):
    ts = np.empty(max(n, 0), np.float32)
    sg = np.empty(max(n, 0) + 1, np.float32)
    c = scheduler_config(**kw)
    rc = load_library().sana_scheduler_schedule_config(ctypes.byref(c), _i(n), _ptr(ts), _ptr(sg))
    if rc != 0:
        raise ValueError("build_sana_scheduler_timesteps rejects this config")
    return ts, sg


def block_tensor_table(block19: Sequence[np.ndarray]) -> List[Optional[np.ndarray]]:
    """Maps the 19 checkpoint tensors of a block (sana_b200.synthetic.BLOCK_TENSORS order)
    to the 26 SanaBlockWeights fields, with the loader's defaults (NULL = zero bias /
    identity norm), as load_block_weights does (transformer.cpp:361-398)."""
    b = list(block19)
    return [b[0], None, None, b[1], None, b[2], None, b[3], None, b[4], b[5], b[6], b[7], b[8], b[9], b[10], b[11],
            b[12], b[13], None, None, b[14], b[15], b[16], b[17], b[18]]


class SanaCuda:
    """One handle of the CUDA library on `device` in `mode` (SANA_MODE_BF16 / _F32)."""

    def __init__(self, device: int = 0, mode: int = SANA_MODE_BF16):
        self.lib = load_library()
        h = ctypes.c_void_p()
        rc = self.lib.sana_cuda_create(_i(device), _i(mode), ctypes.byref(h))
        self.h = h
        if rc != 0:
            msg = self.lib.sana_cuda_last_error(h).decode() if h else "create failed"
            self.close()
            raise SanaError(rc, msg)
        self.mode = mode
        self.dims: Optional[sana_dims] = None
        self._keep = None

    def close(self):
        if getattr(self, "h", None) and self.h:
            self.lib.sana_cuda_destroy(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _call(self, name, *args):
        rc = getattr(self.lib, name)(self.h, *args)
        if rc != 0:
            msg = self.lib.sana_cuda_last_error(self.h).decode()
            if rc == 1:
                raise ValueError(msg)
            raise SanaError(rc, msg)

    @property
    def stream(self) -> int:
        return self.lib.sana_cuda_stream(self.h) or 0

    def synchronize(self):
        self._call("sana_cuda_synchronize")

    def set_cross_qk_norm(self, enable: bool, q_weights=None, k_weights=None, eps: float = 1e-6):
        """Optional RMSNorm of the cross-attention q / k projections (off by default; not in the
        reference). q_weights / k_weights: per-block [hidden] arrays, or None for ones."""
        n = self.dims.n_blocks if self.dims is not None else 0

        def table(ws):
            if ws is None:
                return None
            keep = [_f32(w) for w in ws]
            self._keep_qk = getattr(self, "_keep_qk", []) + keep
            return (_f32p * n)(*[_ptr(w) for w in keep])
        self._call("sana_cuda_set_cross_qk_norm", _i(1 if enable else 0), table(q_weights), table(k_weights), _f(eps))

    def set_wait_limit(self, ns: int):
        """Time limit of the handle's bounded device-side waits (sana_cuda_set_wait_limit)."""
        self._call("sana_cuda_set_wait_limit", ctypes.c_ulonglong(ns))

    def wait_limit(self) -> int:
        self.lib.sana_cuda_wait_limit.restype = ctypes.c_ulonglong
        self.lib.sana_cuda_wait_limit.argtypes = [ctypes.c_void_p]
        return int(self.lib.sana_cuda_wait_limit(self.h))

    def selftest_wait(self, flag_ptr: int, expect: int):
        """One device thread waits for the int at flag_ptr to equal `expect` (bounded)."""
        self._call("sana_cuda_selftest_wait", ctypes.c_void_p(flag_ptr), _i(expect))

    def set_stream(self, stream_ptr: int):
        """Runs later work on the given cudaStream_t (0 restores the handle's own stream)."""
        self._call("sana_cuda_set_stream", ctypes.c_void_p(stream_ptr or None))

    def gemm_device(self, A: int, B: int, M: int, N: int, K: int, out: int, bias: int = 0, act: int = 0):
        vp = ctypes.c_void_p
        self._call("sana_op_gemm_device", vp(A), vp(B), _i(M), _i(N), _i(K), vp(bias) if bias else None, _i(act),
                   vp(out))

    def denoise_loop_ptrs(self, lat: int, B: int, H: int, W: int, enc: int, L: int, Din: int, bias: int, out: int,
                          guidance: float = 4.5, num_steps: int = 20, flow_shift: float = 3.0):
        """sana_cuda_denoise_loop on raw host pointers (e.g. pinned buffers)."""
        vp = ctypes.c_void_p
        self._call("sana_cuda_denoise_loop", vp(lat), _i(B), _i(H), _i(W), vp(enc), _i(L), _i(Din),
                   vp(bias) if bias else None, _f(guidance), _i(num_steps), _f(flow_shift), vp(out))

    def last_launch_count(self) -> int:
        return self.lib.sana_cuda_last_launch_count(self.h)

    def debug_read(self, name: str, count: int, dtype=np.float32, offset_elems: int = 0) -> np.ndarray:
        """A copy of the first `count` elements (after `offset_elems`) of a workspace buffer."""
        out = np.empty(count, dtype)
        isz = out.itemsize
        self._call("sana_cuda_debug_read", name.encode(), ctypes.c_size_t(offset_elems * isz),
                   ctypes.c_size_t(count * isz), out.ctypes.data_as(ctypes.c_void_p), None)
        return out

    # -- weights ------------------------------------------------------------------------
    def upload(self, dims, model16: Sequence[np.ndarray], blocks26: Sequence[Optional[np.ndarray]],
               layout: int = SANA_LAYOUT_TORCH):
        """dims: (n_blocks, hidden, latent_channels, caption_dim, ff_expanded, self_heads, cross_heads)."""
        d = sana_dims(*[int(v) for v in dims])
        keep = [_f32(t) for t in list(model16) + list(blocks26)]
        arr_m = (_f32p * 16)(*[_ptr(t) for t in keep[:16]])
        arr_b = (_f32p * len(blocks26))(*[_ptr(t) for t in keep[16:]])
        self._call("sana_cuda_upload_weights", ctypes.byref(d), arr_m, arr_b, _i(layout))
        self.dims = d

    def upload_checkpoint(self, dims, tensors: Sequence[np.ndarray]):
        """Uploads a synthetic checkpoint list (16 model tensors, 19 per block, PyTorch layout)."""
        nb = int(dims[0])
        blocks: List[Optional[np.ndarray]] = []
        for i in range(nb):
            blocks += block_tensor_table(tensors[16 + 19 * i: 16 + 19 * (i + 1)])
        self.upload(dims, tensors[:16], blocks, SANA_LAYOUT_TORCH)

    def prompt_pairs_device(self, negative, negative_real, positive, positive_real, L: int = 300):
        """sana_cuda_prompt_pairs_device on torch CUDA tensors: negative [pairs, L, hidden],
        positive [pairs, positive_rows, hidden] fp32 -> (enc [2 * pairs, L, hidden],
        bias [2 * pairs, 1, L]) on the device, negatives first."""
        import torch
        pairs, rows, hidden = positive.shape
        nr = (_i * pairs)(*[int(v) for v in negative_real])
        pr = (_i * pairs)(*[int(v) for v in positive_real])
        enc = torch.empty((2 * pairs, L, hidden), dtype=torch.float32, device=positive.device)
        bias = torch.empty((2 * pairs, 1, L), dtype=torch.float32, device=positive.device)
        self._call("sana_cuda_prompt_pairs_device", _i(pairs), ctypes.c_void_p(negative.data_ptr()), nr,
                   ctypes.c_void_p(positive.data_ptr()), _i(rows), pr, _i(hidden), _i(L),
                   ctypes.c_void_p(enc.data_ptr()), ctypes.c_void_p(bias.data_ptr()))
        return enc, bias

    # -- VAE decoder (vae.cpp:243-325) --------------------------------------------------
    def vae_upload(self, dims, tensors):
        """dims: synthetic_vae.VaeDims; tensors: fp32 arrays in its upload order."""
        from .synthetic_vae import dims_struct
        ds = dims_struct(dims)
        arrs = [_f32(t) for t in tensors]
        table = (ctypes.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
        self._call("sana_cuda_vae_upload", ctypes.byref(ds), table)
        self.vae_dims = dims

    def vae_upload_gguf(self, path: str, scaling_factor: float = 0.41407):
        """sana_cuda_vae_upload_gguf: the reference's vae_decoder_weights.gguf; returns the
        VaeDims read from it."""
        from .synthetic_vae import VaeDims, VaeDimsStruct
        ds = VaeDimsStruct()
        self._call("sana_cuda_vae_upload_gguf", os.fsencode(path), _f(scaling_factor), ctypes.byref(ds))
        n = ds.n_blocks
        self.vae_dims = VaeDims(latent_channels=ds.latent_channels, out_channels=ds.out_channels,
                                channels=tuple(ds.blocks[i].channels for i in range(n)),
                                res_blocks=tuple(bool(ds.blocks[i].is_res_block) for i in range(n)),
                                layers=tuple(ds.blocks[i].layers for i in range(n)), head_dim=ds.head_dim,
                                ms_kernel=ds.ms_kernel, scaling_factor=ds.scaling_factor)
        return self.vae_dims

    def vae_decode(self, latents):
        lat = _f32(latents)
        B, _, h, w = lat.shape
        up = self.vae_dims.upscale()
        out = np.empty((B, self.vae_dims.out_channels, h * up, w * up), np.float32)
        self._call("sana_cuda_vae_decode", _ptr(lat), _i(B), _i(h), _i(w), _ptr(out))
        return out

    def vae_decode_device(self, lat_ptr: int, B: int, h: int, w: int, out_ptr: int):
        self._call("sana_cuda_vae_decode_device", ctypes.c_void_p(lat_ptr), _i(B), _i(h), _i(w),
                   ctypes.c_void_p(out_ptr))

    def vae_last_launches(self) -> int:
        return self.lib.sana_cuda_vae_last_launch_count(self.h)

    def upload_gguf(self, model_path: str, caption_path: str, denoiser_path: str, self_heads: int = 36,
                    cross_heads: int = 16):
        """Uploads the reference's three GGUF weight files straight into the device cache;
        returns the dims read from them."""
        d = sana_dims()
        self._call("sana_cuda_upload_gguf", os.fsencode(model_path), os.fsencode(caption_path),
                   os.fsencode(denoiser_path), _i(self_heads), _i(cross_heads), ctypes.byref(d))
        self.dims = d
        return (d.n_blocks, d.hidden, d.latent_channels, d.caption_dim, d.ff_expanded, d.self_heads, d.cross_heads)

    # -- denoiser path (host buffers) ---------------------------------------------------
    def denoise_loop(self, latents, enc, bias, guidance: float = 4.5, num_steps: int = 20, flow_shift: float = 3.0):
        lat, enc, bias = _f32(latents), _f32(enc), _f32(bias)
        B, Cl, H, W = lat.shape
        L, Din = enc.shape[1], enc.shape[2]
        out = np.empty_like(lat)
        self._call("sana_cuda_denoise_loop", _ptr(lat), _i(B), _i(H), _i(W), _ptr(enc), _i(L), _i(Din), _ptr(bias),
                   _f(guidance), _i(num_steps), _f(flow_shift), _ptr(out))
        return out

    def denoise_loop_device(self, lat_ptr: int, B: int, H: int, W: int, enc_ptr: int, L: int, Din: int,
                            bias_ptr: Optional[int], out_ptr: int, guidance: float = 4.5, num_steps: int = 20,
                            flow_shift: float = 3.0):
        vp = ctypes.c_void_p
        self._call("sana_cuda_denoise_loop_device", vp(lat_ptr), _i(B), _i(H), _i(W), vp(enc_ptr), _i(L), _i(Din),
                   vp(bias_ptr) if bias_ptr else None, _f(guidance), _i(num_steps), _f(flow_shift), vp(out_ptr))

    # --- guidance across two GPUs (sana_cuda_cfg_pair_*) --------------------------------------

    def cfg_pair_export(self, max_latent_elems: int) -> bytes:
        """Allocates this GPU's exchange region; returns its 64-byte CUDA IPC handle."""
        buf = ctypes.create_string_buffer(64)
        self._call("sana_cuda_cfg_pair_export", ctypes.c_size_t(max_latent_elems), buf)
        return buf.raw

    def cfg_pair_connect(self, branch: int, peer_handle: bytes):
        """Maps the peer's region; branch 0 runs the unconditional sequences, 1 the conditional."""
        if len(peer_handle) != 64:
            raise ValueError("a peer handle is 64 bytes")
        self._call("sana_cuda_cfg_pair_connect", _i(branch), ctypes.create_string_buffer(peer_handle, 64))

    def cfg_pair_close(self):
        self._call("sana_cuda_cfg_pair_close")

    def denoise_loop_pair_device(self, lat_ptr: int, B: int, H: int, W: int, enc_ptr: int, L: int, Din: int,
                                 bias_ptr: Optional[int], out_ptr: int, guidance: float = 4.5, num_steps: int = 20,
                                 flow_shift: float = 3.0):
        """The loop of this GPU's branch: enc [B, L, Din] / bias [B, 1, L] of that branch."""
        vp = ctypes.c_void_p
        self._call("sana_cuda_denoise_loop_pair_device", vp(lat_ptr), _i(B), _i(H), _i(W), vp(enc_ptr), _i(L),
                   _i(Din), vp(bias_ptr) if bias_ptr else None, _f(guidance), _i(num_steps), _f(flow_shift),
                   vp(out_ptr))

    def profile_loop_device(self, lat_ptr: int, B: int, H: int, W: int, enc_ptr: int, L: int, Din: int,
                            bias_ptr: Optional[int], out_ptr: int, guidance: float = 4.5, num_steps: int = 20,
                            flow_shift: float = 3.0) -> dict:
        """One eager loop with CUDA events around every launch: {kernel class: (launches, ms)}."""
        import json
        vp = ctypes.c_void_p
        buf = ctypes.create_string_buffer(1 << 16)
        self._call("sana_cuda_profile_loop", vp(lat_ptr), _i(B), _i(H), _i(W), vp(enc_ptr), _i(L), _i(Din),
                   vp(bias_ptr) if bias_ptr else None, _f(guidance), _i(num_steps), _f(flow_shift), vp(out_ptr), buf,
                   ctypes.c_size_t(len(buf)))
        return {k: tuple(v) for k, v in json.loads(buf.value.decode()).items()}

    def denoise_step(self, latents, context, bias, guidance, timestep, sigmas, step_index, lower, history):
        """Returns (latents, step_index, lower, history list)."""
        lat = _f32(latents).copy()
        ctx, bias, sg = _f32(context), _f32(bias), _f32(sigmas)
        B, Cl, H, W = lat.shape
        n = lat.size
        hist = np.zeros((2, n), np.float32)
        for i, h in enumerate(history):
            hist[i] = np.asarray(h, np.float32).reshape(-1)
        si, lo, nh = _i(step_index), _i(lower), _i(len(history))
        self._call("sana_cuda_denoise_step", _ptr(lat), _i(B), _i(H), _i(W), _ptr(ctx), _i(ctx.shape[1]), _ptr(bias),
                   _f(guidance), _f(timestep), _ptr(sg), _i(sg.size), ctypes.byref(si), ctypes.byref(lo),
                   _ptr(hist), ctypes.byref(nh))
        return lat, si.value, lo.value, [hist[i].copy() for i in range(nh.value)]

    def time_embed(self, tvals):
        """Timestep embedding + t_block on the device: (emb [S, C], tmod [S, 6C])."""
        t = np.ascontiguousarray(np.asarray(tvals, np.float32).ravel())
        S = t.size
        C = self.dims.hidden
        emb = np.empty((S, C), np.float32)
        tmod = np.empty((S, 6 * C), np.float32)
        self._call("sana_cuda_time_embed", _ptr(t), _i(S), _ptr(emb), _ptr(tmod))
        return emb, tmod

    def forward(self, latents, t, context, bias=None):
        lat, ctx, bias = _f32(latents), _f32(context), _f32(bias)
        S, Cl, H, W = lat.shape
        out = np.empty_like(lat)
        self._call("sana_cuda_forward", _ptr(lat), _i(S), _i(H), _i(W), _f(t), _ptr(ctx), _i(ctx.shape[1]),
                   _ptr(bias), _ptr(out))
        return out

    def block_forward(self, block, x, context, tmod, bias=None):
        x, ctx, tmod, bias = _f32(x), _f32(context), _f32(tmod), _f32(bias)
        S, T, C = x.shape
        outs = [np.empty_like(x) for _ in range(3)]
        self._call("sana_cuda_block_forward", _i(block), _ptr(x), _i(S), _i(T), _ptr(ctx), _i(ctx.shape[1]),
                   _ptr(tmod), _ptr(bias), *[_ptr(o) for o in outs])
        return outs

    def run_model_blocks(self, x, context, tmod, bias=None, begin=0, end=None):
        x, ctx, tmod, bias = _f32(x), _f32(context), _f32(tmod), _f32(bias)
        S, T, C = x.shape
        end = self.dims.n_blocks if end is None else end
        out = np.empty_like(x)
        self._call("sana_cuda_run_model_blocks", _ptr(x), _i(S), _i(T), _ptr(ctx), _i(ctx.shape[1]), _ptr(tmod),
                   _ptr(bias), _i(begin), _i(end), _ptr(out))
        return out

    def project_caption_model(self, enc):
        enc = _f32(enc)
        S, L, Din = enc.shape
        out = np.empty((S, L, self.dims.hidden), np.float32)
        self._call("sana_cuda_project_caption", _ptr(enc), _i(S), _i(L), _i(Din), _ptr(out))
        return out

    # -- single operations (oracle-compatible names) ------------------------------------
    def linear_3d(self, x, w, bias=None):
        x, w, bias = _f32(x), _f32(w), _f32(bias)
        lead = x.shape[:-1]
        K, N = w.shape
        rows = int(np.prod(lead))
        out = np.empty(lead + (N,), np.float32)
        self._call("sana_op_linear", _ptr(x), _i(rows), _i(K), _ptr(w), _ptr(bias), _i(N), _ptr(out))
        return out

    def layer_norm(self, x, eps, gamma=None, beta=None):
        x, gamma, beta = _f32(x), _f32(gamma), _f32(beta)
        C = x.shape[-1]
        out = np.empty_like(x)
        self._call("sana_op_layer_norm", _ptr(x), _i(x.size // C), _i(C), _f(eps), _ptr(gamma), _ptr(beta), _ptr(out))
        return out

    def rms_norm(self, x, eps, weight=None):
        x, weight = _f32(x), _f32(weight)
        C = x.shape[-1]
        out = np.empty_like(x)
        self._call("sana_op_rms_norm", _ptr(x), _i(x.size // C), _i(C), _f(eps), _ptr(weight), _ptr(out))
        return out

    def modulate(self, x, shift, scale):
        x, shift, scale = _f32(x), _f32(shift), _f32(scale)
        B, T, C = x.shape
        out = np.empty_like(x)
        self._call("sana_op_modulate", _ptr(x), _i(B), _i(T), _i(C), _ptr(shift), _ptr(scale), _ptr(out))
        return out

    def linear_attention(self, q, k, v):
        q, k, v = _f32(q), _f32(k), _f32(v)
        B, H, Tq, D = q.shape
        out = np.empty_like(q)
        self._call("sana_op_linear_attention", _ptr(q), _ptr(k), _ptr(v), _i(B), _i(H), _i(Tq), _i(k.shape[2]), _i(D),
                   _ptr(out))
        return out

    def attention(self, q, k, v, bias=None):
        q, k, v, bias = _f32(q), _f32(k), _f32(v), _f32(bias)
        B, H, Tq, D = q.shape
        out = np.empty_like(q)
        self._call("sana_op_attention", _ptr(q), _ptr(k), _ptr(v), _i(B), _i(H), _i(Tq), _i(k.shape[2]), _i(D),
                   _ptr(bias), _ptr(out))
        return out

    def conv1x1(self, x, w, bias=None):
        x, w, bias = _f32(x), _f32(w), _f32(bias)
        B, Cin, H, W = x.shape
        Cout = w.shape[0]
        out = np.empty((B, Cout, H, W), np.float32)
        self._call("sana_op_conv1x1", _ptr(x), _i(B), _i(Cin), _i(H), _i(W), _ptr(w), _ptr(bias), _i(Cout), _ptr(out))
        return out

    def depthwise3x3(self, x, w, bias=None):
        x, w, bias = _f32(x), _f32(w), _f32(bias)
        B, C, H, W = x.shape
        out = np.empty_like(x)
        self._call("sana_op_depthwise3x3", _ptr(x), _i(B), _i(C), _i(H), _i(W), _ptr(w), _ptr(bias), _ptr(out))
        return out

    def glumb_conv(self, x, w_inv, b_inv, w_dw, b_dw, w_pt):
        x, w_inv, b_inv, w_dw, b_dw, w_pt = map(_f32, (x, w_inv, b_inv, w_dw, b_dw, w_pt))
        B, Cin, H, W = x.shape
        E, Cout = w_inv.shape[0], w_pt.shape[0]
        out = np.empty((B, Cout, H, W), np.float32)
        self._call("sana_op_glumb_conv", _ptr(x), _i(B), _i(Cin), _i(H), _i(W), _ptr(w_inv), _ptr(b_inv), _i(E),
                   _ptr(w_dw), _ptr(b_dw), _ptr(w_pt), _i(Cout), _ptr(out))
        return out

    def project_caption(self, enc, w1, b1, w2, b2, norm_w):
        enc, w1, b1, w2, b2, norm_w = map(_f32, (enc, w1, b1, w2, b2, norm_w))
        B, L, Din = enc.shape
        C = w1.shape[1]
        out = np.empty((B, L, C), np.float32)
        self._call("sana_op_project_caption", _ptr(enc), _i(B), _i(L), _i(Din), _ptr(w1), _ptr(b1), _i(C), _ptr(w2),
                   _ptr(b2), _ptr(norm_w), _ptr(out))
        return out

    def attention_block(self, x, wq, bq, wk, bk, wv, bv, wo, bo, heads):
        x, wq, bq, wk, bk, wv, bv, wo, bo = map(_f32, (x, wq, bq, wk, bk, wv, bv, wo, bo))
        B, T, C = x.shape
        out = np.empty_like(x)
        self._call("sana_op_attention_block", _ptr(x), _i(B), _i(T), _i(C), _ptr(wq), _ptr(bq), _ptr(wk), _ptr(bk),
                   _ptr(wv), _ptr(bv), _ptr(wo), _ptr(bo), _i(heads), _ptr(out))
        return out

    def cross_attention_block(self, x, ctx, bias, wq, bq, wk, bk, wv, bv, wo, bo, heads):
        x, ctx, bias, wq, bq, wk, bk, wv, bv, wo, bo = map(_f32, (x, ctx, bias, wq, bq, wk, bk, wv, bv, wo, bo))
        B, T, C = x.shape
        out = np.empty_like(x)
        self._call("sana_op_cross_attention_block", _ptr(x), _i(B), _i(T), _i(C), _ptr(ctx), _i(ctx.shape[1]),
                   _ptr(bias), _ptr(wq), _ptr(bq), _ptr(wk), _ptr(bk), _ptr(wv), _ptr(bv), _ptr(wo), _ptr(bo),
                   _i(heads), _ptr(out))
        return out

    def cfg(self, noise, g):
        noise = _f32(noise)
        B2, Cl, H, W = noise.shape
        out = np.empty((B2 // 2, Cl, H, W), np.float32)
        self._call("sana_op_cfg", _ptr(noise), _i(B2 // 2), _i(Cl), _i(H), _i(W), _f(g), _ptr(out))
        return out

    def scheduler_schedule(self, n: int, flow_shift: float = 3.0):
        return scheduler_schedule(n, flow_shift)

    def scheduler_convert(self, sigmas, step_index, model_output, sample):
        sg, mo, x = _f32(sigmas), _f32(model_output).reshape(-1), _f32(sample).reshape(-1)
        out = np.empty_like(x)
        self._call("sana_scheduler_convert", _ptr(sg), _i(sg.size), _i(step_index), _ptr(mo), _ptr(x), _i(x.size),
                   _ptr(out))
        return out

    def scheduler_update(self, order, sigmas, step_index, m0, m1, sample):
        sg, x = _f32(sigmas), _f32(sample).reshape(-1)
        m0 = _f32(m0).reshape(-1)
        m1 = _f32(m1).reshape(-1) if m1 is not None else None
        out = np.empty_like(x)
        self._call("sana_scheduler_update", _i(order), _ptr(sg), _i(sg.size), _i(step_index), _ptr(m0), _ptr(m1),
                   _ptr(x), _i(x.size), _ptr(out))
        return out

    def scheduler_step(self, sigmas, step_index, lower, hist, model_output, sample):
        sg, mo, x = _f32(sigmas), _f32(model_output).reshape(-1), _f32(sample).reshape(-1)
        n = x.size
        h = np.zeros((2, n), np.float32)
        for i, a in enumerate(hist):
            h[i] = np.asarray(a, np.float32).reshape(-1)
        si, lo, nh = _i(step_index), _i(lower), _i(len(hist))
        out = np.empty_like(x)
        self._call("sana_scheduler_step", _ptr(sg), _i(sg.size), ctypes.byref(si), ctypes.byref(lo), _ptr(h),
                   ctypes.byref(nh), _ptr(mo), _ptr(x), _i(n), _ptr(out))
        return out, [h[i].copy() for i in range(nh.value)], lo.value

    def scheduler_step_config(self, config: dict, sigmas, step_index, lower, hist, model_output, sample):
        """step_sana_scheduler with a config (dict of sana_scheduler_config fields):
        returns (new_sample, new_history [oldest first], new_lower_count, new_step_index)."""
        c = scheduler_config(**config)
        sg, mo, x = _f32(sigmas), _f32(model_output).reshape(-1), _f32(sample).reshape(-1)
        n = x.size
        h = np.zeros((2, n), np.float32)
        for i, a in enumerate(hist):
            h[i] = np.asarray(a, np.float32).reshape(-1)
        si, lo, nh = _i(step_index), _i(lower), _i(len(hist))
        out = np.empty_like(x)
        self._call("sana_scheduler_step_config", ctypes.byref(c), _ptr(sg), _i(sg.size), ctypes.byref(si),
                   ctypes.byref(lo), _ptr(h), ctypes.byref(nh), _ptr(mo), _ptr(x), _i(n), _ptr(out))
        return out, [h[i].copy() for i in range(nh.value)], lo.value, si.value

    def scheduler_update_config(self, config: dict, order, sigmas, step_index, m0, m1, sample):
        c = scheduler_config(**config)
        sg, x = _f32(sigmas), _f32(sample).reshape(-1)
        m0 = _f32(m0).reshape(-1)
        m1 = _f32(m1).reshape(-1) if m1 is not None else None
        out = np.empty_like(x)
        self._call("sana_scheduler_update_config", ctypes.byref(c), _i(order), _ptr(sg), _i(sg.size), _i(step_index),
                   _ptr(m0), _ptr(m1), _ptr(x), _i(x.size), _ptr(out))
        return out

    def denoise_loop_config(self, config: dict, latents, enc, bias, guidance: float = 4.5, num_steps: int = 20):
        c = scheduler_config(**config)
        lat, enc, bias = _f32(latents), _f32(enc), _f32(bias)
        B, Cl, H, W = lat.shape
        L, Din = enc.shape[1], enc.shape[2]
        out = np.empty_like(lat)
        self._call("sana_cuda_denoise_loop_config", ctypes.byref(c), _ptr(lat), _i(B), _i(H), _i(W), _ptr(enc),
                   _i(L), _i(Din), _ptr(bias), _f(guidance), _i(num_steps), _ptr(out))
        return out

    def denoise_step_config(self, config: dict, latents, context, bias, guidance, timestep, sigmas, step_index,
                            lower, history):
        """Returns (latents, step_index, lower, history list)."""
        c = scheduler_config(**config)
        lat = _f32(latents).copy()
        ctx, bias, sg = _f32(context), _f32(bias), _f32(sigmas)
        B, Cl, H, W = lat.shape
        n = lat.size
        hist = np.zeros((2, n), np.float32)
        for i, h in enumerate(history):
            hist[i] = np.asarray(h, np.float32).reshape(-1)
        si, lo, nh = _i(step_index), _i(lower), _i(len(history))
        self._call("sana_cuda_denoise_step_config", ctypes.byref(c), _ptr(lat), _i(B), _i(H), _i(W), _ptr(ctx),
                   _i(ctx.shape[1]), _ptr(bias), _f(guidance), _f(timestep), _ptr(sg), _i(sg.size), ctypes.byref(si),
                   ctypes.byref(lo), _ptr(hist), ctypes.byref(nh))
        return lat, si.value, lo.value, [hist[i].copy() for i in range(nh.value)]

    # -- model handle compatible with the checkers' model() ------------------------------
    def model(self, tensors, n_blocks, C, Cl, Din, E, self_heads, cross_heads):
        self.upload_checkpoint((n_blocks, C, Cl, Din, E, self_heads, cross_heads), tensors)
        return _GpuModel(self)


class _GpuModel:
    """Model-level methods under the checkers' names (oracle/oracle.py _CpuModel)."""

    def __init__(self, g: SanaCuda):
        self.g = g

    def block_forward(self, block, x, ctx, tmod, bias=None):
        return self.g.block_forward(block, x, ctx, tmod, bias)

    def run_model_blocks(self, x, ctx, tmod, bias=None, begin=0, end=None):
        return self.g.run_model_blocks(x, ctx, tmod, bias, begin, end)

    def project_caption(self, enc):
        return self.g.project_caption_model(enc)

    def time_embed(self, tvals):
        return self.g.time_embed(tvals)

    def forward_nocfg(self, latents, t, ctx, bias=None):
        return self.g.forward(latents, t, ctx, bias)

    def denoise(self, latents, enc, bias, guidance, num_steps, run_steps=None):
        assert run_steps is None or run_steps == num_steps
        return self.g.denoise_loop(latents, enc, bias, guidance, num_steps)
