"""Python host layer over libb200diff.so (the sm_100a diffusion hot-path library).

Mirrors the reference's entry points for this path:
  * ``VibeVoiceDiffusionHead``   ~ VibeVoiceDiffusionHeadWeightsRuntime + sample_vibevoice_speech_latents
    (include/engine/models/vibevoice/diffusion_head.h:58-97, diffusion_sampler.h:23-26)
  * ``vv_schedule``              ~ VibeVoiceDPMSolverScheduler timesteps / step coefficients
Everything runs through the C ABI declared in include/b200diff.h.  There is no
CPU fallback: if the library or a B200 is missing the calls raise.

This directory name contains a dot, so load it by path, e.g.
``importlib.util.spec_from_file_location("audiocpp_b200", ".../audio.cpp_b200/__init__.py")``.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Dict, Iterable, Optional, Sequence, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libb200diff.so")

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_BF16 = 0, 1, 8, 30
EPI_F32, EPI_CT, EPI_SWIGLU, EPI_RESID = 0, 1, 2, 3

STATUS = {0: "ok", -1: "EINVAL", -2: "ECUDA", -3: "ENOMEM", -4: "ESTATE", -5: "ENONFINITE", -6: "ETIMEOUT",
          -7: "ENODEV"}

EXPORTED = ["b2d_create", "b2d_destroy", "b2d_last_error", "b2d_sync", "b2d_version", "b2d_vv_schedule",
            "b2d_vv_head_load", "b2d_vv_predict", "b2d_vv_sample", "b2d_vv_sample_device", "b2d_q8_0_dequantize",
            "b2d_storage_resolve", "b2d_tensor_bytes", "b2d_tensor_convert", "b2d_gemm", "b2d_gemm_stream", "b2d_gemm_splitk_noalloc", "b2d_gemm_splitk_noalloc_status", "b2d_gemm_splitk_noalloc_selftest_timeout", "b2d_dit_load", "b2d_dit_sample", "b2d_dit_sample_device", "b2d_attention", "b2d_torch_randn", "b2d_selftest_wait_timeout",
            "b2d_sa3_load", "b2d_sa3_sample", "b2d_sa3_sample_device", "b2d_oobleck_load", "b2d_oobleck_decode",
            "b2d_oobleck_decode_device", "b2d_vvdec_load", "b2d_vvdec_decode", "b2d_vvdec_decode_device",
            "b2d_saocond_load", "b2d_saocond_encode", "b2d_saocond_encode_device",
            "b2d_vvlm_load", "b2d_vvlm_prefill", "b2d_vvlm_step", "b2d_vvlm_prefill_device", "b2d_vvlm_step_device"]


class B2DError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__("%s (%s)" % (message, STATUS.get(status, status)))
        self.status = status


class TensorView(C.Structure):
    _fields_ = [("name", C.c_char_p), ("ggml_type", C.c_int32), ("ndim", C.c_int32), ("dims", C.c_int64 * 4),
                ("data", C.c_void_p), ("nbytes", C.c_size_t)]


class HeadConfig(C.Structure):
    _fields_ = [("hidden_size", C.c_int64), ("latent_size", C.c_int64), ("head_layers", C.c_int64),
                ("head_ffn_ratio", C.c_float), ("rms_norm_eps", C.c_float), ("ddpm_num_steps", C.c_int64)]


class VvStep(C.Structure):
    _fields_ = [("timestep", C.c_int64), ("sigma", C.c_float), ("sigma_next", C.c_float), ("alpha_s", C.c_float),
                ("sigma_s", C.c_float), ("sample_coeff", C.c_float), ("d0_coeff", C.c_float),
                ("inv_r0", C.c_float), ("order", C.c_int32)]


class DitConfig(C.Structure):
    _fields_ = [("embed_dim", C.c_int64), ("depth", C.c_int64), ("num_heads", C.c_int64),
                ("cond_token_dim", C.c_int64), ("global_cond_dim", C.c_int64), ("io_channels", C.c_int64),
                ("prompt_max_length", C.c_int64)]


class DitRequest(C.Structure):
    _fields_ = [("batch", C.c_int64), ("latent_tokens", C.c_int64), ("steps", C.c_int64), ("noise", C.c_void_p),
                ("padding_mask", C.c_void_p), ("cross_positive", C.c_void_p), ("cross_negative", C.c_void_p),
                ("global_cond", C.c_void_p), ("sigma_min", C.c_float), ("sigma_max", C.c_float), ("rho", C.c_float),
                ("cfg_scale", C.c_float), ("apg_scale", C.c_float), ("sampler", C.c_int32), ("schedule", C.c_void_p),
                ("seed", C.c_uint64), ("rng_offset_blocks", C.POINTER(C.c_uint64)),
                ("rng_multiprocessor_count", C.c_int64), ("rng_max_threads_per_multiprocessor", C.c_int64),
                ("rng_batch_total", C.c_int64), ("rng_batch_first", C.c_int64)]


class Sa3Config(C.Structure):
    _fields_ = [("embed_dim", C.c_int64), ("depth", C.c_int64), ("num_heads", C.c_int64), ("cond_dim", C.c_int64),
                ("global_cond_dim", C.c_int64), ("local_add_cond_dim", C.c_int64), ("num_memory_tokens", C.c_int64),
                ("io_channels", C.c_int64), ("prompt_max_length", C.c_int64), ("differential_attention", C.c_int32)]


class Sa3Request(C.Structure):
    _fields_ = [("batch", C.c_int64), ("latent_tokens", C.c_int64), ("schedule_points", C.c_int64),
                ("noise", C.c_void_p), ("padding_mask", C.c_void_p), ("schedule", C.c_void_p),
                ("cross_positive", C.c_void_p), ("cross_negative", C.c_void_p), ("negative_mask", C.c_void_p),
                ("global_cond", C.c_void_p), ("local_add", C.c_void_p), ("cfg_scale", C.c_float),
                ("apg_scale", C.c_float), ("sampler", C.c_int32), ("seed", C.c_uint64),
                ("rng_offset_blocks", C.POINTER(C.c_uint64)), ("rng_multiprocessor_count", C.c_int64),
                ("rng_max_threads_per_multiprocessor", C.c_int64), ("rng_batch_total", C.c_int64),
                ("rng_batch_first", C.c_int64)]


class OobleckConfig(C.Structure):
    _fields_ = [("latent_dim", C.c_int64), ("channels", C.c_int64), ("audio_channels", C.c_int64),
                ("n_blocks", C.c_int32), ("c_mults", C.c_int64 * 8), ("strides", C.c_int64 * 8)]


class VvdecConfig(C.Structure):
    _fields_ = [("vae_dim", C.c_int64), ("n_filters", C.c_int64), ("n_stages", C.c_int32),
                ("ratios", C.c_int64 * 8), ("depths", C.c_int64 * 8), ("disable_last_norm", C.c_int32),
                ("eps", C.c_float)]


class SaoCondConfig(C.Structure):
    _fields_ = [("hidden", C.c_int64), ("layers", C.c_int64), ("heads", C.c_int64), ("head_dim", C.c_int64),
                ("intermediate", C.c_int64), ("vocab", C.c_int64), ("prompt_max_length", C.c_int64),
                ("eps", C.c_float)]


class VvlmConfig(C.Structure):
    _fields_ = [("hidden", C.c_int64), ("intermediate", C.c_int64), ("heads", C.c_int64), ("kv_heads", C.c_int64),
                ("head_dim", C.c_int64), ("layers", C.c_int64), ("vocab", C.c_int64), ("max_positions", C.c_int64),
                ("eps", C.c_float), ("rope_theta", C.c_float)]


SA3_SAMPLERS = {"": 0, "pingpong": 0, "euler": 1}

SAMPLERS = {"dpmpp-2m": 0, "dpmpp-3m-sde": 1, "": 2, "euler": 2, "pingpong": 2}


_lib = None


def lib() -> C.CDLL:
    """Loads the in-tree library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("libb200diff.so is not built; run python audio.cpp_b200/build.py")
        L = C.CDLL(LIB_PATH)
        P, I64, F, I32 = C.c_void_p, C.c_int64, C.c_float, C.c_int32
        L.b2d_create.argtypes = [C.c_int, C.POINTER(P)]
        L.b2d_destroy.argtypes = [P]
        L.b2d_destroy.restype = None
        L.b2d_last_error.argtypes = [P]
        L.b2d_last_error.restype = C.c_char_p
        L.b2d_version.restype = C.c_char_p
        L.b2d_sync.argtypes = [P, P]
        L.b2d_vv_schedule.argtypes = [I64, I64, C.POINTER(VvStep)]
        L.b2d_vv_head_load.argtypes = [P, C.POINTER(HeadConfig), C.POINTER(TensorView), I32]
        L.b2d_vv_predict.argtypes = [P, P, I64, I64, F, P, I64, P, P]
        L.b2d_vv_sample.argtypes = [P, P, P, P, I64, I64, F, P, P]
        L.b2d_vv_sample_device.argtypes = [P, P, P, P, I64, I64, F, P, P]
        L.b2d_q8_0_dequantize.argtypes = [P, P, I64, I64, P, P]
        L.b2d_gemm.argtypes = [P, I32, P, P, I64, I64, I64, I32, I32, P, P, I64, P, I64, P, I64, P]
        L.b2d_storage_resolve.argtypes = [I32, C.POINTER(TensorView)]
        L.b2d_storage_resolve.restype = I32
        L.b2d_tensor_bytes.argtypes = [I32, C.POINTER(I64), I32]
        L.b2d_tensor_bytes.restype = C.c_size_t
        L.b2d_tensor_convert.argtypes = [C.POINTER(TensorView), I32, P, C.c_size_t]
        L.b2d_gemm_stream.argtypes = [P, I32, P, P, I32, I64, I64, I64, I32, I32, I32, P, P, I64, P, I64, P, I64, P]
        L.b2d_gemm_splitk_noalloc.argtypes = [I32, P, P, I64, I64, I64, I32, I32, P, P, I64, P, C.c_char_p,
                                              C.c_size_t]
        L.b2d_gemm_splitk_noalloc_status.argtypes = [P, C.c_char_p, C.c_size_t]
        L.b2d_gemm_splitk_noalloc_selftest_timeout.argtypes = [C.c_uint32, P, C.c_char_p, C.c_size_t]
        L.b2d_attention.argtypes = [P, I32, P, I64, I64, P, P, I64, I64, P, I64, I64, I32, I32, I32, I32, I32, P]
        L.b2d_selftest_wait_timeout.argtypes = [P, C.c_uint32, P]
        L.b2d_torch_randn.argtypes = [P, I32, C.c_uint64, C.c_uint64, I64, I64, I64, I32, P, P]
        L.b2d_dit_load.argtypes = [P, C.POINTER(DitConfig), C.POINTER(TensorView), I32]
        L.b2d_dit_sample.argtypes = [P, C.POINTER(DitRequest), P, P]
        L.b2d_dit_sample_device.argtypes = [P, C.POINTER(DitRequest), P, P]
        L.b2d_sa3_load.argtypes = [P, C.POINTER(Sa3Config), C.POINTER(TensorView), I32]
        L.b2d_sa3_sample.argtypes = [P, C.POINTER(Sa3Request), P, P]
        L.b2d_sa3_sample_device.argtypes = [P, C.POINTER(Sa3Request), P, P]
        L.b2d_oobleck_load.argtypes = [P, C.POINTER(OobleckConfig), C.POINTER(TensorView), I32]
        L.b2d_oobleck_decode.argtypes = [P, P, I64, I64, P, P]
        L.b2d_oobleck_decode_device.argtypes = [P, P, I64, I64, P, P]
        L.b2d_vvdec_load.argtypes = [P, C.POINTER(VvdecConfig), C.POINTER(TensorView), I32]
        L.b2d_vvdec_decode.argtypes = [P, P, I64, P, P]
        L.b2d_vvdec_decode_device.argtypes = [P, P, I64, P, P]
        L.b2d_saocond_load.argtypes = [P, C.POINTER(SaoCondConfig), C.POINTER(TensorView), I32]
        L.b2d_saocond_encode.argtypes = [P, P, P, P, I64, P, P, P, P]
        L.b2d_saocond_encode_device.argtypes = [P, P, P, P, I64, P, P, P, P]
        L.b2d_vvlm_load.argtypes = [P, C.POINTER(VvlmConfig), C.POINTER(TensorView), I32]
        L.b2d_vvlm_prefill.argtypes = [P, P, I64, P, P, P]
        L.b2d_vvlm_step.argtypes = [P, P, P, P, P]
        L.b2d_vvlm_prefill_device.argtypes = [P, P, I64, P, P, P]
        L.b2d_vvlm_step_device.argtypes = [P, P, P, P, P]
        _lib = L
    return _lib


STORAGE_NATIVE, STORAGE_F32, STORAGE_F16, STORAGE_BF16, STORAGE_Q8_0 = 0, 1, 2, 3, 13


def convert_tensor(ggml_type: int, dims, payload: np.ndarray, storage: int):
    """The reference weight store's storage-type selection + conversion of one checkpoint tensor (host).
    Returns (ggml_type, payload bytes as uint8)."""
    payload = np.ascontiguousarray(payload)
    v = TensorView()
    v.name = b"t"
    v.ggml_type = ggml_type
    v.ndim = len(dims)
    for j, d in enumerate(dims):
        v.dims[j] = d
    v.data = payload.ctypes.data
    v.nbytes = payload.nbytes
    target = lib().b2d_storage_resolve(storage, C.byref(v))
    if target < 0:
        raise B2DError(-1, "unsupported storage type %d" % storage)
    nbytes = lib().b2d_tensor_bytes(target, v.dims, v.ndim)
    out = np.empty(nbytes, np.uint8)
    st = lib().b2d_tensor_convert(C.byref(v), target, out.ctypes.data, nbytes)
    if st != 0:
        raise B2DError(st, "tensor conversion failed")
    return target, out


def version() -> str:
    return lib().b2d_version().decode()


def vv_schedule(ddpm_num_steps: int, steps: int) -> Sequence[VvStep]:
    """VibeVoiceDPMSolverScheduler(ddpm_num_steps).set_timesteps(steps) tables + step coefficients (host only)."""
    out = (VvStep * steps)()
    st = lib().b2d_vv_schedule(ddpm_num_steps, steps, out)
    if st != 0:
        raise B2DError(st, "VibeVoice scheduler requires positive timestep counts")
    return list(out)


def _ptr(a) -> int:
    """Host numpy array or torch tensor (host or device) -> raw address."""
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


class Context:
    """One device context (b2d_ctx).  Not thread-safe; one per GPU."""

    def __init__(self, device: int = 0):
        self._h = C.c_void_p()
        st = lib().b2d_create(device, C.byref(self._h))
        if st != 0:
            raise B2DError(st, "b2d_create(%d) failed: no usable sm_100 device" % device)
        self.device = device

    def close(self) -> None:
        if self._h:
            lib().b2d_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, status: int) -> None:
        if status != 0:
            raise B2DError(status, lib().b2d_last_error(self._h).decode())

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def sync(self, stream: int = 0) -> None:
        self.check(lib().b2d_sync(self._h, C.c_void_p(stream)))

    # ---------------------------------------------------------- kernel entries
    def q8_0_dequantize(self, q8_dev: int, rows: int, k: int, out_dev: int, stream: int = 0) -> None:
        self.check(lib().b2d_q8_0_dequantize(self._h, C.c_void_p(q8_dev), rows, k, C.c_void_p(out_dev),
                                             C.c_void_p(stream)))

    def selftest_wait_timeout(self, polls: int, stream: int = 0) -> None:
        """Runs a kernel whose bounded wait must expire; raises B2DError(B2D_ETIMEOUT)."""
        self.check(lib().b2d_selftest_wait_timeout(self._h, polls, C.c_void_p(stream)))

    def torch_randn(self, out_dev: int, count: int, seed: int, offset: int = 0, layout: int = 0, sms: int = 1,
                    max_threads: int = 256, bf16: bool = False, stream: int = 0) -> None:
        """torch-CUDA-compatible normals into a device float buffer (layout 0 per-index, 1 TensorIterator)."""
        self.check(lib().b2d_torch_randn(self._h, layout, seed, offset, count, sms, max_threads, int(bf16),
                                         C.c_void_p(out_dev), C.c_void_p(stream)))

    def attention(self, q: int, q_row: int, q_seq: int, k: int, v: int, kv_row: int, kv_seq: int, o: int,
                  o_row: int, o_seq: int, lq: int, lk: int, heads: int, kv_rep: int = 1, nseq: int = 1,
                  bf16: bool = False, stream: int = 0) -> None:
        self.check(lib().b2d_attention(self._h, int(bf16), C.c_void_p(q), q_row, q_seq, C.c_void_p(k), C.c_void_p(v),
                                       kv_row, kv_seq, C.c_void_p(o), o_row, o_seq, lq, lk, heads, kv_rep, nseq,
                                       C.c_void_p(stream)))

    def gemm(self, a_dev: int, b_dev: int, m: int, n: int, k: int, *, bf16: bool = False, epilogue: int = EPI_F32,
             bn: int = 256, bias: int = 0, out: int = 0, ldo: int = 0, resid: int = 0, ldr: int = 0, gate: int = 0,
             ldg: int = 0, stream: int = 0) -> None:
        self.check(lib().b2d_gemm(self._h, int(bf16), C.c_void_p(a_dev), C.c_void_p(b_dev), m, n, k, epilogue, bn,
                                  C.c_void_p(bias or None), C.c_void_p(out or None), ldo, C.c_void_p(resid or None),
                                  ldr, C.c_void_p(gate or None), ldg, C.c_void_p(stream)))


    def gemm_stream(self, a_dev: int, w_dev: int, m: int, n: int, k: int, *, w_type: int, bf16: bool = False,
                    epilogue: int = EPI_F32, bn: int = 0, split: int = 1, bias: int = 0, out: int = 0, ldo: int = 0,
                    resid: int = 0, ldr: int = 0, gate: int = 0, ldg: int = 0, stream: int = 0) -> None:
        """Weight-streaming GEMM (M <= 128); w_type = ggml type id of W on the device (1 F16, 30 BF16, 8 Q8_0);
        bn = 0 plans the tile width and K split itself."""
        self.check(lib().b2d_gemm_stream(self._h, int(bf16), C.c_void_p(a_dev), C.c_void_p(w_dev), w_type, m, n, k,
                                         epilogue, bn, split, C.c_void_p(bias or None), C.c_void_p(out or None), ldo,
                                         C.c_void_p(resid or None), ldr, C.c_void_p(gate or None), ldg,
                                         C.c_void_p(stream)))


WeightSpec = Tuple[str, int, Tuple[int, ...], np.ndarray]  # (name, ggml type, dims, raw payload)


def _views(specs):
    """(name, ggml_type, dims, payload) list -> (TensorView array, keep-alive list)."""
    specs = list(specs)
    views = (TensorView * len(specs))()
    keep = []
    for i, (name, gtype, dims, payload) in enumerate(specs):
        payload = np.ascontiguousarray(payload)
        nb = name.encode()
        keep += [payload, nb]
        views[i].name = nb
        views[i].ggml_type = gtype
        views[i].ndim = len(dims)
        for j, dd in enumerate(dims):
            views[i].dims[j] = dd
        views[i].data = payload.ctypes.data
        views[i].nbytes = payload.nbytes
    return views, keep


class StableAudioDiT:
    """FoundationRfDitRuntime (include/engine/models/stable_audio/foundation/rf_dit.h:73-106) on a B200 context.

    ``weights``: (name, ggml_type, dims, payload) with the GGUF names ``model.model.*``."""

    def __init__(self, ctx: Context, embed_dim: int = 1536, depth: int = 24, num_heads: int = 24,
                 cond_token_dim: int = 768, global_cond_dim: int = 1536, io_channels: int = 64,
                 prompt_max_length: int = 128, weights: Iterable[WeightSpec] = ()):
        self.ctx = ctx
        self.cfg = DitConfig(embed_dim, depth, num_heads, cond_token_dim, global_cond_dim, io_channels,
                             prompt_max_length)
        views, keep = _views(weights)
        ctx.check(lib().b2d_dit_load(ctx.handle, C.byref(self.cfg), views, len(keep) // 2))

    def _request(self, noise, padding_mask, cross_positive, cross_negative, global_cond, steps, sigma_min,
                 sigma_max, rho, cfg_scale, apg_scale, sampler="dpmpp-2m", schedule=None, seed=0, rng_offset=0,
                 rng_policy=(1, 256), rng_batch=(0, 0)):
        b, _, t = noise.shape
        self._offset = C.c_uint64(rng_offset)
        return DitRequest(b, t, steps, _ptr(noise), _ptr(padding_mask), _ptr(cross_positive),
                          _ptr(cross_negative) if cross_negative is not None else None, _ptr(global_cond),
                          sigma_min, sigma_max, rho, cfg_scale, apg_scale, SAMPLERS[sampler],
                          _ptr(schedule) if schedule is not None else None, seed, C.pointer(self._offset),
                          rng_policy[0], rng_policy[1], rng_batch[1], rng_batch[0])

    @property
    def rng_offset_blocks(self) -> int:
        """TensorIterator Philox offset after the last call (the reference's rng_offset_blocks out-parameter)."""
        return int(self._offset.value)

    def sample(self, noise, padding_mask, cross_positive, cross_negative, global_cond, steps=100, sigma_min=0.01,
               sigma_max=100.0, rho=1.0, cfg_scale=7.0, apg_scale=1.0, out=None, stream: int = 0,
               sampler="dpmpp-2m", schedule=None, seed=0, rng_offset=0, rng_policy=(1, 256), rng_batch=(0, 0)):
        """Host arrays (numpy / pinned torch) -> latents [B, 64, T].  rng_batch = (first prompt, prompts in the
        whole batch) when this call is one data-parallel shard of a batched request (noise as the batched call)."""
        arrs = [np.ascontiguousarray(a, np.float32) if isinstance(a, np.ndarray) else a
                for a in (noise, padding_mask, cross_positive, cross_negative, global_cond, schedule)]
        rq = self._request(*arrs[:5], steps, sigma_min, sigma_max, rho, cfg_scale, apg_scale, sampler, arrs[5], seed,
                           rng_offset, rng_policy, rng_batch)
        if out is None:
            out = np.empty(arrs[0].shape, np.float32)
        self.ctx.check(lib().b2d_dit_sample(self.ctx.handle, C.byref(rq), C.c_void_p(_ptr(out)), C.c_void_p(stream)))
        return out

    def sample_device(self, noise, padding_mask, cross_positive, cross_negative, global_cond, out, steps=100,
                      sigma_min=0.01, sigma_max=100.0, rho=1.0, cfg_scale=7.0, apg_scale=1.0, stream: int = 0,
                      sampler="dpmpp-2m", schedule=None, seed=0, rng_offset=0, rng_policy=(1, 256), rng_batch=(0, 0)):
        rq = self._request(noise, padding_mask, cross_positive, cross_negative, global_cond, steps, sigma_min,
                           sigma_max, rho, cfg_scale, apg_scale, sampler, schedule, seed, rng_offset, rng_policy,
                           rng_batch)
        self.ctx.check(lib().b2d_dit_sample_device(self.ctx.handle, C.byref(rq), C.c_void_p(_ptr(out)),
                                                   C.c_void_p(stream)))
        return out


class StableAudio3DiT:
    """StableAudioRfDitRuntime (include/engine/models/stable_audio/rf_dit.h:78-100) on a B200 context: the
    Stable Audio 3 rectified-flow DiT with memory tokens, local-add conditioning and optional differential
    attention.  ``weights``: (name, ggml_type, dims, payload) with the GGUF names ``model.model.*``."""

    def __init__(self, ctx: Context, embed_dim: int, depth: int, num_heads: int, cond_dim: int,
                 global_cond_dim: int, local_add_cond_dim: int, num_memory_tokens: int, prompt_max_length: int,
                 differential_attention: bool = False, io_channels: int = 64, weights: Iterable[WeightSpec] = ()):
        self.ctx = ctx
        self.cfg = Sa3Config(embed_dim, depth, num_heads, cond_dim, global_cond_dim, local_add_cond_dim,
                             num_memory_tokens, io_channels, prompt_max_length, int(bool(differential_attention)))
        self._offset = C.c_uint64(0)
        views, keep = _views(weights)
        ctx.check(lib().b2d_sa3_load(ctx.handle, C.byref(self.cfg), views, len(keep) // 2))

    @property
    def rng_offset_blocks(self) -> int:
        """TensorIterator Philox offset after the last call (the reference's rng_offset_blocks out-parameter)."""
        return int(self._offset.value)

    def _request(self, noise, padding_mask, schedule, cross_positive, cross_negative, negative_mask, global_cond,
                 local_add, cfg_scale, apg_scale, sampler, seed, rng_offset, rng_policy, rng_batch=(0, 0)):
        b, _, t = noise.shape
        self._offset = C.c_uint64(rng_offset)
        opt = lambda a: _ptr(a) if a is not None else None  # noqa: E731
        return Sa3Request(b, t, schedule.shape[-1], _ptr(noise), _ptr(padding_mask), _ptr(schedule),
                          _ptr(cross_positive), opt(cross_negative), opt(negative_mask), _ptr(global_cond),
                          _ptr(local_add), cfg_scale, apg_scale, SA3_SAMPLERS.get(sampler, -1), seed,
                          C.pointer(self._offset), rng_policy[0], rng_policy[1], rng_batch[1], rng_batch[0])

    def sample(self, noise, padding_mask, schedule, cross_positive, cross_negative, negative_mask, global_cond,
               local_add, cfg_scale=7.0, apg_scale=1.0, sampler="pingpong", seed=0, rng_offset=0,
               rng_policy=(1, 256), out=None, stream: int = 0, rng_batch=(0, 0)):
        """Host arrays (numpy / pinned torch) -> latents [B, 64, T].  rng_batch = (first prompt, prompts in the
        whole batch) when this call is one data-parallel shard of a batched request (noise as the batched call)."""
        arrs = [np.ascontiguousarray(a, np.float32) if isinstance(a, np.ndarray) else a
                for a in (noise, padding_mask, schedule, cross_positive, cross_negative, negative_mask, global_cond,
                          local_add)]
        rq = self._request(*arrs, cfg_scale, apg_scale, sampler, seed, rng_offset, rng_policy, rng_batch)
        if out is None:
            out = np.empty(arrs[0].shape, np.float32)
        self.ctx.check(lib().b2d_sa3_sample(self.ctx.handle, C.byref(rq), C.c_void_p(_ptr(out)), C.c_void_p(stream)))
        return out

    def sample_device(self, noise, padding_mask, schedule, cross_positive, cross_negative, negative_mask,
                      global_cond, local_add, out, cfg_scale=7.0, apg_scale=1.0, sampler="pingpong", seed=0,
                      rng_offset=0, rng_policy=(1, 256), stream: int = 0, rng_batch=(0, 0)):
        """Device tensors (torch CUDA) -> out (device), asynchronous on `stream`."""
        rq = self._request(noise, padding_mask, schedule, cross_positive, cross_negative, negative_mask, global_cond,
                           local_add, cfg_scale, apg_scale, sampler, seed, rng_offset, rng_policy, rng_batch)
        self.ctx.check(lib().b2d_sa3_sample_device(self.ctx.handle, C.byref(rq), C.c_void_p(_ptr(out)),
                                                   C.c_void_p(stream)))
        return out


class OobleckDecoder:
    """OobleckAutoencoderRuntime's decode half (include/engine/models/stable_audio/foundation/oobleck_autoencoder.h:
    71-96) on a B200 context.  ``weights``: (name, ggml_type, dims, payload) with the names
    ``pretransform.model.decoder.layers.*``."""

    def __init__(self, ctx: Context, latent_dim: int, channels: int, c_mults, strides, audio_channels: int = 2,
                 weights: Iterable[WeightSpec] = ()):
        self.ctx = ctx
        self.cfg = OobleckConfig(latent_dim, channels, audio_channels, len(strides))
        for i, (m, s) in enumerate(zip(c_mults, strides)):
            self.cfg.c_mults[i] = m
            self.cfg.strides[i] = s
        self.hop = int(np.prod(strides))
        self.audio_channels = audio_channels
        views, keep = _views(weights)
        ctx.check(lib().b2d_oobleck_load(ctx.handle, C.byref(self.cfg), views, len(keep) // 2))

    def decode(self, latents, out=None, stream: int = 0):
        """Host latents [B, latent_dim, T] -> audio [B, T x hop, audio_channels]."""
        latents = np.ascontiguousarray(latents, np.float32) if isinstance(latents, np.ndarray) else latents
        b, _, t = latents.shape
        if out is None:
            out = np.empty((b, t * self.hop, self.audio_channels), np.float32)
        self.ctx.check(lib().b2d_oobleck_decode(self.ctx.handle, _ptr(latents), b, t, _ptr(out), C.c_void_p(stream)))
        return out

    def decode_device(self, latents, out, stream: int = 0):
        """Device latents -> device audio, asynchronous on `stream`."""
        b, _, t = latents.shape
        self.ctx.check(lib().b2d_oobleck_decode_device(self.ctx.handle, _ptr(latents), b, t, _ptr(out),
                                                       C.c_void_p(stream)))
        return out


class VibeVoiceAcousticDecoder:
    """VibeVoiceTokenizerWeightsRuntime::decode_acoustic (include/engine/models/vibevoice/tokenizer_audio.h:94-140)
    on a B200 context.  ``weights``: (name, ggml_type, dims, payload) with the names
    ``model.acoustic_tokenizer.decoder.*``; ``depths`` in encoder order, ``ratios`` = decoder_ratios."""

    def __init__(self, ctx: Context, vae_dim: int, n_filters: int, ratios, depths, disable_last_norm: bool = True,
                 eps: float = 1e-5, weights: Iterable[WeightSpec] = ()):
        self.ctx = ctx
        self.cfg = VvdecConfig(vae_dim, n_filters, len(depths))
        for i, r in enumerate(ratios):
            self.cfg.ratios[i] = r
        for i, d in enumerate(depths):
            self.cfg.depths[i] = d
        self.cfg.disable_last_norm = int(bool(disable_last_norm))
        self.cfg.eps = eps
        self.hop = int(np.prod(ratios))
        views, keep = _views(weights)
        ctx.check(lib().b2d_vvdec_load(ctx.handle, C.byref(self.cfg), views, len(keep) // 2))

    def decode(self, latents, out=None, stream: int = 0):
        """Host latents [frames, vae_dim] -> mono samples [frames x hop]."""
        latents = np.ascontiguousarray(latents, np.float32) if isinstance(latents, np.ndarray) else latents
        frames = latents.shape[0]
        if out is None:
            out = np.empty(frames * self.hop, np.float32)
        self.ctx.check(lib().b2d_vvdec_decode(self.ctx.handle, _ptr(latents), frames, _ptr(out), C.c_void_p(stream)))
        return out

    def decode_device(self, latents, out, stream: int = 0):
        self.ctx.check(lib().b2d_vvdec_decode_device(self.ctx.handle, _ptr(latents), latents.shape[0], _ptr(out),
                                                     C.c_void_p(stream)))
        return out


class StableAudioConditioner:
    """FoundationConditionerRuntime (include/engine/models/stable_audio/foundation/conditioner.h:43-66) on a B200
    context: T5-base + the seconds number conditioners.  ``weights``: (name, ggml_type, dims, payload) with the
    names ``shared.weight``, ``encoder.*`` and ``conditioner.conditioners.*``."""

    def __init__(self, ctx: Context, hidden: int, layers: int, heads: int, head_dim: int, intermediate: int,
                 vocab: int, prompt_max_length: int, eps: float = 1e-6, weights: Iterable[WeightSpec] = ()):
        self.ctx = ctx
        self.cfg = SaoCondConfig(hidden, layers, heads, head_dim, intermediate, vocab, prompt_max_length, eps)
        views, keep = _views(weights)
        ctx.check(lib().b2d_saocond_load(ctx.handle, C.byref(self.cfg), views, len(keep) // 2))

    def encode_one(self, input_ids, attention_mask, normalized_seconds, stream: int = 0):
        """Host ids / mask [B, P], seconds [B] -> (cross [B, P + 2, d], cross_mask [B, P + 2], global [B, 2 d])."""
        ids = np.ascontiguousarray(input_ids, np.int32)
        mask = np.ascontiguousarray(attention_mask, np.float32)
        secs = np.ascontiguousarray(normalized_seconds, np.float32)
        b, p = ids.shape
        d = self.cfg.hidden
        cross = np.empty((b, p + 2, d), np.float32)
        cmask = np.empty((b, p + 2), np.float32)
        glob = np.empty((b, 2 * d), np.float32)
        self.ctx.check(lib().b2d_saocond_encode(self.ctx.handle, _ptr(ids), _ptr(mask), _ptr(secs), b, _ptr(cross),
                                                _ptr(cmask), _ptr(glob), C.c_void_p(stream)))
        return cross, cmask, glob

    def encode(self, prompt_ids, prompt_mask, normalized_seconds, negative_ids=None, negative_mask=None,
               stream: int = 0):
        """FoundationConditionerRuntime::encode (src/models/stable_audio/foundation/conditioner.cpp:411-420): the
        prompt batch and, when given, the negative prompt batch, both with the batch's normalized total seconds.
        Returns {"positive": (cross, cross_mask, global), "negative": (...) or None}."""
        out = {"positive": self.encode_one(prompt_ids, prompt_mask, normalized_seconds, stream), "negative": None}
        if negative_ids is not None and len(negative_ids) > 0:
            out["negative"] = self.encode_one(negative_ids, negative_mask, normalized_seconds, stream)
        return out


class VibeVoiceLanguageModel:
    """VibeVoiceDecoderWeightsRuntime's prefill / cached step (include/engine/models/vibevoice/decoder.h:106-143) on a
    B200 context; one KV cache per context.  ``weights``: the ``model.language_model.*`` tensors."""

    def __init__(self, ctx: Context, hidden: int, intermediate: int, heads: int, kv_heads: int, head_dim: int,
                 layers: int, vocab: int, max_positions: int, eps: float = 1e-6, rope_theta: float = 1e6,
                 weights: Iterable[WeightSpec] = ()):
        self.ctx = ctx
        self.cfg = VvlmConfig(hidden, intermediate, heads, kv_heads, head_dim, layers, vocab, max_positions, eps,
                              rope_theta)
        views, keep = _views(weights)
        ctx.check(lib().b2d_vvlm_load(ctx.handle, C.byref(self.cfg), views, len(keep) // 2))

    def prefill(self, embeddings, stream: int = 0):
        """Host embeddings [steps, hidden] -> (logits [vocab], last_hidden [hidden]) of the last position."""
        e = np.ascontiguousarray(embeddings, np.float32)
        logits = np.empty(self.cfg.vocab, np.float32)
        hidden = np.empty(self.cfg.hidden, np.float32)
        self.ctx.check(lib().b2d_vvlm_prefill(self.ctx.handle, _ptr(e), e.shape[0], _ptr(logits), _ptr(hidden),
                                              C.c_void_p(stream)))
        return logits, hidden

    def step(self, embedding, stream: int = 0):
        e = np.ascontiguousarray(embedding, np.float32).reshape(-1)
        logits = np.empty(self.cfg.vocab, np.float32)
        hidden = np.empty(self.cfg.hidden, np.float32)
        self.ctx.check(lib().b2d_vvlm_step(self.ctx.handle, _ptr(e), _ptr(logits), _ptr(hidden), C.c_void_p(stream)))
        return logits, hidden

    def prefill_device(self, embeddings, logits, hidden, stream: int = 0):
        """Device embeddings [steps, hidden] -> device logits [vocab] and hidden [hidden], asynchronous on `stream`
        (torch CUDA tensors, fp32, contiguous)."""
        self.ctx.check(lib().b2d_vvlm_prefill_device(self.ctx.handle, _ptr(embeddings), embeddings.shape[0],
                                                     _ptr(logits), _ptr(hidden), C.c_void_p(stream)))

    def step_device(self, embedding, logits, hidden, stream: int = 0):
        """One cached position from a device embedding [hidden]; outputs as prefill_device."""
        self.ctx.check(lib().b2d_vvlm_step_device(self.ctx.handle, _ptr(embedding), _ptr(logits), _ptr(hidden),
                                                  C.c_void_p(stream)))


class VibeVoiceDiffusionHead:
    """VibeVoiceDiffusionHeadWeightsRuntime on a B200 context.

    ``weights`` is an iterable of (name, ggml_type, dims, payload) with the GGUF
    tensor names ``model.prediction_head.*`` and raw stored bytes.
    """

    def __init__(self, ctx: Context, hidden_size: int, head_layers: int = 4, head_ffn_ratio: float = 3.0,
                 latent_size: int = 64, rms_norm_eps: float = 1e-5, ddpm_num_steps: int = 1000,
                 weights: Iterable[WeightSpec] = ()):
        self.ctx = ctx
        self.hidden_size, self.latent_size = hidden_size, latent_size
        self.ddpm_num_steps = ddpm_num_steps
        cfg = HeadConfig(hidden_size, latent_size, head_layers, head_ffn_ratio, rms_norm_eps, ddpm_num_steps)
        specs = list(weights)
        views = (TensorView * len(specs))()
        keep = []
        for i, (name, gtype, dims, payload) in enumerate(specs):
            payload = np.ascontiguousarray(payload)
            keep.append(payload)
            nb = name.encode()
            keep.append(nb)
            views[i].name = nb
            views[i].ggml_type = gtype
            views[i].ndim = len(dims)
            for j, d in enumerate(dims):
                views[i].dims[j] = d
            views[i].data = payload.ctypes.data
            views[i].nbytes = payload.nbytes
        ctx.check(lib().b2d_vv_head_load(ctx.handle, C.byref(cfg), views, len(specs)))

    def predict(self, noisy: np.ndarray, timestep: float, condition: np.ndarray) -> np.ndarray:
        noisy = np.ascontiguousarray(noisy, np.float32)
        condition = np.ascontiguousarray(condition, np.float32)
        frames = noisy.shape[0]
        out = np.empty((frames, self.latent_size), np.float32)
        self.ctx.check(lib().b2d_vv_predict(self.ctx.handle, _ptr(noisy), frames, noisy.shape[1], float(timestep),
                                            _ptr(condition), condition.shape[1], _ptr(out), None))
        return out

    def sample(self, positive_condition, negative_condition, initial_speech, steps: int, cfg: float,
               out=None, stream: int = 0):
        """Host buffers (numpy or pinned torch CPU tensors) -> latents [B, latent] (sync)."""
        batch = positive_condition.shape[0]
        if out is None:
            out = np.empty((batch, self.latent_size), np.float32)
        self.ctx.check(lib().b2d_vv_sample(self.ctx.handle, _ptr(positive_condition), _ptr(negative_condition),
                                           _ptr(initial_speech), batch, steps, float(cfg), _ptr(out),
                                           C.c_void_p(stream)))
        return out

    def sample_device(self, positive_condition, negative_condition, initial_speech, steps: int, cfg: float, out,
                      stream: int = 0):
        """Device tensors (torch CUDA) -> out (device), asynchronous on `stream`."""
        batch = positive_condition.shape[0]
        self.ctx.check(lib().b2d_vv_sample_device(self.ctx.handle, _ptr(positive_condition),
                                                  _ptr(negative_condition), _ptr(initial_speech), batch, steps,
                                                  float(cfg), _ptr(out), C.c_void_p(stream)))
        return out
