"""Launchers for the reference's own CUDA kernels (kernels/sam.cu of apiplant/sam-rs), compiled by
oracle/build_ref_cuda.py into oracle/_ref/sam.cubin.

TEST INFRASTRUCTURE ONLY. It is used by tests/ and by bench.py's reference arm, to run the reference's
code itself on the GPU: its relpos_softmax, qkv_split, bias_residual and bias_gelu kernels, and its CUDA
attention path. The product package never imports this module.

The module is loaded through the CUDA driver API (cuModuleLoad / cuLaunchKernel), as candle's
custom-module loader does, into torch's current context. Launch configurations follow the reference's host
code:
  * relpos_softmax: one block per score row; threads = n rounded up to 32, at most 256;
    ITEMS = ceil(n / threads) rounded up to a power of two; dynamic shared memory (hd + h + w) floats
    (src/kernels.rs:1117-1131).
  * the elementwise kernels: blocks of 256 threads, ceil(total / 256) blocks, at most 65536
    (src/kernels.rs:1104-1106).
  * the attention path: bmm(relpos_softmax(bmm(q, kt)), v) (src/sam1/encoder.rs:81). The reference's bmm
    is candle's cuBLAS matmul in the I/O dtype with f32 accumulation; torch.bmm does the same here, with
    TF32 and reduced-precision reductions switched off.
"""
import ctypes
import os

from . import build_ref_cuda

_SUF = {"float32": "f32", "float16": "f16", "bfloat16": "bf16"}
_THREADS, _MAXI = 256, 32  # src/kernels.rs:1080-1081


class RefCudaError(RuntimeError):
    pass


class RefCuda:
    """The reference's kernels in torch's current CUDA context (device of the tensors passed in)."""

    def __init__(self, path=None):
        path = path or build_ref_cuda.OUT
        if not os.path.exists(path):
            raise RefCudaError(f"{path} not built (the reference's kernels/sam.cu was not present at build time)")
        self.cu = ctypes.CDLL("libcuda.so.1")
        vp, u = ctypes.c_void_p, ctypes.c_uint
        self.cu.cuInit.argtypes = [u]
        self.cu.cuModuleLoad.argtypes = [ctypes.POINTER(vp), ctypes.c_char_p]
        self.cu.cuModuleGetFunction.argtypes = [ctypes.POINTER(vp), vp, ctypes.c_char_p]
        self.cu.cuLaunchKernel.argtypes = [vp, u, u, u, u, u, u, u, vp, ctypes.POINTER(vp), ctypes.POINTER(vp)]
        self._check(self.cu.cuInit(0), "cuInit")
        import torch
        torch.cuda.init()
        torch.empty(1, device="cuda")  # make torch's primary context current on this thread
        self.mod = ctypes.c_void_p()
        self._check(self.cu.cuModuleLoad(ctypes.byref(self.mod), path.encode()), "cuModuleLoad")
        self.funcs = {}

    def _check(self, rc, what):
        if rc != 0:
            raise RefCudaError(f"{what} failed with CUresult {rc}")

    def _func(self, name):
        f = self.funcs.get(name)
        if f is None:
            f = ctypes.c_void_p()
            self._check(self.cu.cuModuleGetFunction(ctypes.byref(f), self.mod, name.encode()),
                        f"cuModuleGetFunction({name})")
            self.funcs[name] = f
        return f

    def _launch(self, name, grid, block, smem, args, stream):
        holders = []
        for a in args:
            if isinstance(a, ctypes._SimpleCData):
                holders.append(a)
            else:
                raise TypeError(a)
        params = (ctypes.c_void_p * len(holders))(*[ctypes.addressof(h) for h in holders])
        self._check(self.cu.cuLaunchKernel(self._func(name), grid, 1, 1, block, 1, 1, smem, ctypes.c_void_p(stream),
                                           params, None),
                    f"cuLaunchKernel({name})")

    @staticmethod
    def _suffix(t):
        return _SUF[str(t.dtype).replace("torch.", "")]

    @staticmethod
    def _stream():
        import torch
        return torch.cuda.current_stream().cuda_stream

    def relpos_softmax(self, s, q, table, h, w, scale):
        """The reference's RelposSoftmax (src/kernels.rs:1108-1131, kernels/sam.cu:44-106): s [rows, n] (any
        leading shape), q [rows, hd] matching, table [(2h-1)+(2w-1), hd]; returns the probabilities."""
        import torch
        n = h * w
        hd = q.shape[-1]
        assert s.is_contiguous() and q.is_contiguous() and table.is_contiguous()
        assert s.dtype == q.dtype == table.dtype and s.shape[-1] == n and n <= _THREADS * _MAXI
        rows = s.numel() // n
        assert q.numel() == rows * hd and table.shape == ((2 * h - 1) + (2 * w - 1), hd)
        threads = min((n + 31) // 32 * 32, _THREADS)
        items = 1
        while items < -(-n // threads):
            items *= 2
        out = torch.empty_like(s)
        self._launch(f"relpos_softmax_i{items}_{self._suffix(s)}", rows, threads, (hd + h + w) * 4,
                     [ctypes.c_void_p(s.data_ptr()), ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(table.data_ptr()),
                      ctypes.c_void_p(out.data_ptr()), ctypes.c_int(h), ctypes.c_int(w), ctypes.c_int(hd),
                      ctypes.c_float(scale)], self._stream())
        return out

    def _grid(self, total):
        return min(-(-total // 256), 1 << 16)

    def qkv_split(self, y, bias, n, nh, hd):
        """The reference's QkvSplit (src/kernels.rs:1186-1198): y [windows*n, 3*nh*hd] + bias -> q, kt, v."""
        import torch
        assert y.is_contiguous() and bias.is_contiguous() and y.dtype == bias.dtype
        total = y.numel()
        out = torch.empty(total, dtype=y.dtype, device=y.device)
        self._launch(f"qkv_split_{self._suffix(y)}", self._grid(total), 256, 0,
                     [ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(bias.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                      ctypes.c_long(total), ctypes.c_int(n), ctypes.c_int(nh), ctypes.c_int(hd)], self._stream())
        plane = total // 3
        bh = plane // (n * hd)
        return (out[:plane].view(bh, n, hd), out[plane:2 * plane].view(bh, hd, n), out[2 * plane:].view(bh, n, hd))

    def bias_residual(self, res, y, bias):
        """The reference's BiasResidual (kernels/sam.cu:130-135): res + y + bias[col]."""
        import torch
        assert res.shape == y.shape and res.is_contiguous() and y.is_contiguous()
        total, c = y.numel(), bias.numel()
        out = torch.empty_like(y)
        self._launch(f"bias_residual_{self._suffix(y)}", self._grid(total), 256, 0,
                     [ctypes.c_void_p(res.data_ptr()), ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(bias.data_ptr()),
                      ctypes.c_void_p(out.data_ptr()), ctypes.c_long(total), ctypes.c_int(c)], self._stream())
        return out

    def bias_gelu(self, y, bias):
        """The reference's BiasGelu (kernels/sam.cu:137-143): erf GELU of y + bias[col]."""
        import torch
        assert y.is_contiguous()
        total, c = y.numel(), bias.numel()
        out = torch.empty_like(y)
        self._launch(f"bias_gelu_{self._suffix(y)}", self._grid(total), 256, 0,
                     [ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(bias.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                      ctypes.c_long(total), ctypes.c_int(c)], self._stream())
        return out

    @staticmethod
    def matmul(a, b):
        """candle's CUDA matmul as the reference uses it (src/kernels.rs:919-924): cuBLAS in the I/O dtype
        with f32 accumulation, no TF32 and no reduced-precision reductions."""
        import torch
        mm = torch.backends.cuda.matmul
        saved = (mm.allow_tf32, mm.allow_fp16_reduced_precision_reduction, mm.allow_bf16_reduced_precision_reduction)
        mm.allow_tf32 = False
        mm.allow_fp16_reduced_precision_reduction = False
        mm.allow_bf16_reduced_precision_reduction = False
        try:
            return torch.matmul(a, b)
        finally:
            mm.allow_tf32, mm.allow_fp16_reduced_precision_reduction, mm.allow_bf16_reduced_precision_reduction = saved

    def attention(self, q, kt, v, table, h, w, scale):
        """The reference's CUDA attention path, src/sam1/encoder.rs:81:
        bmm(relpos_softmax(bmm(q, kt), q, table), v), every intermediate in the I/O dtype."""
        s = self.matmul(q, kt)
        p = self.relpos_softmax(s, q, table, h, w, scale)
        del s
        return self.matmul(p, v)
