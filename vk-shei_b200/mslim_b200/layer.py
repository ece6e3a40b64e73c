"""One Llama-3-shaped decoder layer on the device, sequenced as the reference's
GPU runtime runs it (GpuLlm::run_layer, src/gpu_llm/mod.rs:2118-2329, and the
batched prefill, src/gpu_llm/prefill.rs:292-435) and with the per-token
arithmetic of the CPU decoder (forward_token, src/native_cpu_adapter.rs:
486-577):

    n = RMSNorm(x); q, k, v = n Wq^T, n Wk^T, n Wv^T; RoPE(q, k); append K/V;
    a = attention(q, K, V); x = x + a Wo^T;
    n = RMSNorm(x); x = x + SwiGLU(n Wg^T, n Wu^T) Wd^T

Projections are cuBLAS GEMMs through torch.matmul (bf16 operands, fp32
accumulation, one bf16 rounding per output, like the CPU matvec's
round_bf16(sum)); RMSNorm, RoPE (+ the K/V page append), attention, the
residual adds and SwiGLU are kernels of libmslim_cuda.so.

The K/V of a layer live either in a dense token-major cache
([capacity][KVH][D], the GPU runtime's workspace caches) or in ColdStore-exact
pages ([n_pages][KVH][page_tokens][D] behind a page table, the layout of
src/cold_store.rs:725-742).  Prefill attention reads the batch's own K/V in
both modes (BatchKernels::attention); decode reads the cache or the pages, with
the same kernel code, so the two modes return identical bits.
"""
from __future__ import annotations

import dataclasses

import numpy as np

from . import attention as _att


@dataclasses.dataclass(frozen=True)
class LayerSpec:
    """Llama-3-8B layer shape."""
    hidden: int = 4096
    intermediate: int = 14336
    query_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    eps: float = 1e-5
    theta: float = 500000.0

    @property
    def q_dim(self) -> int:
        return self.query_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim


WEIGHT_NAMES = ("input_norm", "wq", "wk", "wv", "wo", "post_norm", "wg", "wu", "wd")


def weight_shapes(spec: LayerSpec) -> dict:
    h, i = spec.hidden, spec.intermediate
    return {"input_norm": (h,), "wq": (spec.q_dim, h), "wk": (spec.kv_dim, h), "wv": (spec.kv_dim, h),
            "wo": (h, spec.q_dim), "post_norm": (h,), "wg": (i, h), "wu": (i, h), "wd": (h, i)}


def random_layer_weights(spec: LayerSpec, seed: int, std: float = 0.02) -> dict:
    """Random-init weights as bf16 bits: projections N(0, std) rounded to
    bf16; RMSNorm weights one (the Llama initialisation)."""
    from .workloads import bf16_bits
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in weight_shapes(spec).items():
        if name.endswith("norm"):
            out[name] = np.full(shape, 0x3F80, np.uint16)  # bf16 1.0
        else:
            out[name] = bf16_bits((rng.standard_normal(shape, dtype=np.float32) * np.float32(std)))
    return out


def embedding_rows(ids: np.ndarray, hidden: int, seed: int) -> np.ndarray:
    """Rows of an N(0, 1) bf16 embedding table for token `ids`: row i is drawn
    from its own generator (seed, i), so the 128 256 x hidden table never has
    to be materialised."""
    from .workloads import bf16_bits
    rows = np.empty((len(ids), hidden), np.uint16)
    for r, i in enumerate(np.asarray(ids, np.int64)):
        rows[r] = bf16_bits(np.random.default_rng([seed, int(i)]).standard_normal(hidden, dtype=np.float32))
    return rows


class DeviceLayer:
    """One decoder layer's weights on the device plus its K/V store."""

    def __init__(self, spec: LayerSpec, weights: dict, capacity: int, kv_mode: str = "dense",
                 page_tokens: int = 256, page_seed: int = 0, device=None):
        import torch
        if kv_mode not in ("dense", "coldstore"):
            raise ValueError("kv_mode is 'dense' or 'coldstore'")
        # one rounding per output from an fp32 accumulator, as the CPU matvec
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
        self.torch = torch
        self.spec = spec
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.w = {k: torch.from_numpy(np.ascontiguousarray(v, np.uint16).view(np.int16)).to(self.device)
                  .view(torch.bfloat16) for k, v in weights.items()}
        self.geometry = _att.AttentionGeometry.new(spec.query_heads, spec.kv_heads, spec.head_dim)
        self.rope_cfg = _att.RopeKernelConfig(theta=spec.theta)
        self.capacity = capacity
        self.kv_mode = kv_mode
        bf = torch.bfloat16
        if kv_mode == "dense":
            self.k_cache = torch.zeros((capacity, spec.kv_heads, spec.head_dim), dtype=bf, device=self.device)
            self.v_cache = torch.zeros_like(self.k_cache)
        else:
            self.page_tokens = page_tokens
            self.max_pages = (capacity + page_tokens - 1) // page_tokens
            # physical pages in a random order, as a ColdStore file fills them
            perm = np.random.default_rng(page_seed).permutation(self.max_pages).astype(np.int32)
            self.page_table = torch.from_numpy(perm.reshape(1, -1)).to(self.device)
            self.k_pool = torch.zeros((self.max_pages, spec.kv_heads, page_tokens, spec.head_dim), dtype=bf,
                                      device=self.device)
            self.v_pool = torch.zeros_like(self.k_pool)
        # the paged decode sizes its split partials by the page table's reach
        reach = capacity if kv_mode == "dense" else self.max_pages * self.page_tokens
        ws = _att.decode_workspace_bytes(self.geometry, 1, reach)
        self.workspace = torch.zeros(max(ws, 16), dtype=torch.uint8, device=self.device)
        self.position = 0

    # ---- the steps shared by prefill and decode
    def _norm(self, x, weight):
        out = self.torch.empty_like(x)
        _att.rmsnorm(x, weight, out, x.shape[0], self.spec.hidden, self.spec.eps)
        return out

    def _project(self, x, name):
        return self.torch.matmul(x, self.w[name].t())

    def _mlp_residual(self, x, attn):
        s, t = self.spec, self.torch
        o = self._project(attn.reshape(x.shape[0], s.q_dim), "wo")
        _att.residual_add(x, o, x, x.numel())
        n = self._norm(x, self.w["post_norm"])
        g = self._project(n, "wg")
        u = self._project(n, "wu")
        _att.swiglu(g, u, g, g.numel())
        d = self._project(g, "wd")
        _att.residual_add(x, d, x, x.numel())
        return x

    def prefill(self, x):
        """x: bf16 [T][hidden] layer input of the next T positions (from an
        empty cache).  Returns (layer output, post-RoPE q, post-RoPE k, v,
        attention output), all bf16 device tensors."""
        s, t = self.spec, self.torch
        T = x.shape[0]
        if self.position != 0 or T > self.capacity:
            raise ValueError("prefill starts from an empty cache and must fit its capacity")
        x = x.clone()
        n = self._norm(x, self.w["input_norm"])
        q, k, v = self._project(n, "wq"), self._project(n, "wk"), self._project(n, "wv")
        q_r = t.empty_like(q)
        k_r = t.empty_like(k)
        _att.rope(q, q_r, T, s.query_heads, s.head_dim, 0, self.rope_cfg)
        _att.rope(k, k_r, T, s.kv_heads, s.head_dim, 0, self.rope_cfg)
        if self.kv_mode == "dense":
            self.k_cache[:T] = k_r.view(T, s.kv_heads, s.head_dim)
            self.v_cache[:T] = v.view(T, s.kv_heads, s.head_dim)
        else:
            q_pages = t.empty_like(q)
            _att.rope_append_paged(self.geometry, q, q_pages, k, v, T, 0, self.rope_cfg, self.k_pool,
                                   self.v_pool, self.max_pages, self.page_tokens, self.page_table,
                                   self.max_pages)
            if not t.equal(q_pages.view(t.int16), q_r.view(t.int16)):
                raise _att.BackendFailure("RoPE of the page-append path differs from mslim_cuda_rope")
        attn = t.empty_like(q_r)
        _att.prefill_causal(self.geometry, q_r, k_r, v, attn, T, 0)
        x = self._mlp_residual(x, attn)
        self.position = T
        return x, q_r, k_r, v, attn

    def decode(self, x):
        """x: bf16 [1][hidden] layer input of the token at the next position."""
        s, t = self.spec, self.torch
        p = self.position
        if p >= self.capacity:
            raise ValueError("K/V capacity exceeded")
        x = x.clone()
        n = self._norm(x, self.w["input_norm"])
        q, k, v = self._project(n, "wq"), self._project(n, "wk"), self._project(n, "wv")
        q_r = t.empty_like(q)
        attn = t.empty_like(q)
        seq = t.tensor([p + 1], dtype=t.int32, device=self.device)
        if self.kv_mode == "dense":
            k_r = t.empty_like(k)
            _att.rope(q, q_r, 1, s.query_heads, s.head_dim, p, self.rope_cfg)
            _att.rope(k, k_r, 1, s.kv_heads, s.head_dim, p, self.rope_cfg)
            self.k_cache[p] = k_r.view(s.kv_heads, s.head_dim)
            self.v_cache[p] = v.view(s.kv_heads, s.head_dim)
            _att.decode_dense(self.geometry, q_r, self.k_cache, self.v_cache, seq, 1, self.capacity,
                              self.workspace, attn)
        else:
            pos = t.tensor([p], dtype=t.int32, device=self.device)
            _att.rope_append_decode_paged(self.geometry, q, q_r, k, v, pos, 1, self.rope_cfg, self.k_pool,
                                          self.v_pool, self.max_pages, self.page_tokens, self.page_table,
                                          self.max_pages)
            _att.decode_paged(self.geometry, q_r, self.k_pool, self.v_pool, self.max_pages, self.page_tokens,
                              self.page_table, self.max_pages, seq, 1, self.workspace, attn)
        x = self._mlp_residual(x, attn)
        self.position = p + 1
        return x, q_r, attn

    def canonical_kv(self):
        """(K, V) of the committed tokens as device tensors [kv_heads][tokens][head_dim],
        the logical KV digest order, read from whichever store this layer uses."""
        t, s, T = self.torch, self.spec, self.position
        k = t.empty((s.kv_heads, T, s.head_dim), dtype=t.bfloat16, device=self.device)
        v = t.empty_like(k)
        if self.kv_mode == "dense":
            _att.kv_canonical_dense(self.k_cache, s.kv_heads, s.head_dim, T, k)
            _att.kv_canonical_dense(self.v_cache, s.kv_heads, s.head_dim, T, v)
        else:
            for pool, dst in ((self.k_pool, k), (self.v_pool, v)):
                _att.kv_canonical_paged(pool, self.max_pages, s.kv_heads, self.page_tokens, s.head_dim,
                                        self.page_table[0], self.max_pages, T, dst)
        return k, v

    def logical_kv_sha256(self) -> str:
        """The adapters' validation digest over this one layer's K/V state
        (src/gpu_llm/mod.rs:1981-2023): equal for the dense and the
        ColdStore-exact store when they hold the same bf16 K/V."""
        from .digest import LogicalKvHasher, device_tensor_bytes
        hasher = LogicalKvHasher(self.position)
        k, v = self.canonical_kv()
        hasher.add(device_tensor_bytes(self.torch, k), device_tensor_bytes(self.torch, v))
        if _att.device_status(self.device.index or 0) != 0:
            raise _att.ShapeMismatch("a page id outside the pool while reading the K/V state")
        return hasher.hexdigest()
