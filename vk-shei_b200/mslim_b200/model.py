"""A Llama-3-8B-shaped decoder ("C5") on one or
more B200s, tensor-parallel by KV-head group.

Per layer and rank (TP world W, rank r): the rank owns KV heads
[r*KVH/W, (r+1)*KVH/W) and their query heads (GQA mapping qh / (QH/KVH) kept),
so attention needs no exchange; q/k/v projections are column slices, the
o-projection is row-parallel and its partial sums meet in one NCCL all-reduce
(sum, bf16, tokens x hidden) over NVLink.  The MLP is either replicated on
every rank (mlp="replicated": exactly one all-reduce per layer, the MLP's
FLOPs and weight bytes do not scale) or sharded (mlp="sharded": gate/up
column-parallel, down row-parallel, a second all-reduce; everything scales).

Sequencing follows the reference GPU runtime: prefill through the batched
kernels (src/gpu_llm/prefill.rs), decode through run_layer
(src/gpu_llm/mod.rs:2118-2329), then the final norm, the tied lm_head and the
greedy argmax with the CPU path's tie rule (native_cpu_adapter.rs:579-587).
Weights are random: projections and the tied embedding N(0, 0.02), RMSNorm
weights one; each layer's full tensors come from a device generator seeded by
(seed, layer), so every rank slices its shard of the same model.
"""
from __future__ import annotations

import dataclasses

from . import attention as _att
from .layer import LayerSpec


@dataclasses.dataclass(frozen=True)
class ModelSpec:
    layer: LayerSpec = LayerSpec()
    layers: int = 32
    vocab: int = 128256
    std: float = 0.02


class SectionTimer:
    """CUDA events around each step of a forward, summed per kind (gemm,
    attention, collective, elementwise) or per named op once the stream has
    been synchronised.  Each section carries the op's algorithmic bytes (what
    it must move at least: weights, K/V, activations in and out) and the link
    they cross ("hbm", or "nvlink" for the peer reads of a reduction)."""

    def __init__(self, torch):
        self.torch = torch
        self.marks = []

    def __call__(self, kind, op=None, nbytes=0, kernel=None, link="hbm"):
        return _Section(self, kind, op or kind, int(nbytes), kernel or op or kind, link)

    def totals_ms(self) -> dict:
        out = {}
        for sec, a, b in self.marks:
            out[sec.kind] = out.get(sec.kind, 0.0) + a.elapsed_time(b)
        return out

    def per_op(self) -> list:
        """One entry per named op: sections (launches of the op), device ms,
        algorithmic bytes, heaviest first."""
        acc = {}
        for sec, a, b in self.marks:
            e = acc.setdefault(sec.op, {"op": sec.op, "kernel": sec.kernel, "kind": sec.kind, "link": sec.link,
                                        "launches": 0, "ms": 0.0, "bytes": 0})
            e["launches"] += 1
            e["ms"] += a.elapsed_time(b)
            e["bytes"] += sec.nbytes
        return sorted(acc.values(), key=lambda e: -e["ms"])


class _Section:
    def __init__(self, timer, kind, op, nbytes, kernel, link):
        self.timer, self.kind, self.op, self.nbytes, self.kernel, self.link = timer, kind, op, nbytes, kernel, link

    def __enter__(self):
        t = self.timer.torch
        self.a = t.cuda.Event(enable_timing=True)
        self.b = t.cuda.Event(enable_timing=True)
        self.a.record()

    def __exit__(self, *exc):
        self.b.record()
        self.timer.marks.append((self, self.a, self.b))
        return False


class _NoSection:
    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


_NO_SECTION = _NoSection()


def shard_argmax_key(torch, bits, local_ids, vocab_lo: int):
    """One int64 per row ordering a vocabulary shard's maximum: the
    f32::total_cmp key of its bf16 value (bits, int16) above its global index,
    so the largest key wins and, among equal values, the larger index (the CPU
    path's last-maximal-index rule, native_cpu_adapter.rs:582-587)."""
    b = bits.to(torch.int32)
    key = torch.where(b < 0, b ^ 0x7FFF, b)
    return (key.to(torch.int64) << 32) | (local_ids.to(torch.int64) + vocab_lo)


def pick_shard_argmax(torch, every):
    """every: int64 [ranks][rows] of shard_argmax_key -> int32 global token ids."""
    return (every.max(dim=0).values & 0xFFFFFFFF).to(torch.int32)


class DeviceModel:
    def __init__(self, spec: ModelSpec, batch: int, capacity: int, seed: int = 5, tp_rank: int = 0,
                 tp_world: int = 1, mlp: str = "sharded", kv_mode: str = "dense", page_tokens: int = 256,
                 group=None, device=None, decode_gemm: str = "cublas", fuse_qkv: bool = False):
        import torch
        L = spec.layer
        if L.kv_heads % tp_world or L.intermediate % tp_world:
            raise ValueError("KV heads and the MLP width must divide by the tensor-parallel world")
        if mlp not in ("sharded", "replicated"):
            raise ValueError("mlp is 'sharded' or 'replicated'")
        if kv_mode not in ("dense", "coldstore"):
            raise ValueError("kv_mode is 'dense' or 'coldstore'")
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
        self.torch, self.spec = torch, spec
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.rank, self.world, self.group = tp_rank, tp_world, group
        self.mlp, self.kv_mode = mlp, kv_mode
        if decode_gemm not in ("own", "cublas"):
            raise ValueError("decode_gemm is 'own' (mslim_cuda_gemv) or 'cublas'")
        self.decode_gemm = decode_gemm
        self.fuse_qkv = fuse_qkv
        self.batch, self.capacity = batch, capacity
        self.kvh = L.kv_heads // tp_world
        self.qh = L.query_heads // tp_world
        self.geometry = _att.AttentionGeometry.new(self.qh, self.kvh, L.head_dim)
        self.rope_cfg = _att.RopeKernelConfig(theta=L.theta)
        bf = torch.bfloat16
        dev = self.device
        D = L.head_dim
        q0, q1 = tp_rank * self.qh * D, (tp_rank + 1) * self.qh * D
        k0, k1 = tp_rank * self.kvh * D, (tp_rank + 1) * self.kvh * D
        inter = L.intermediate if mlp == "replicated" else L.intermediate // tp_world
        i0 = 0 if mlp == "replicated" else tp_rank * inter

        def normal(g, shape):
            return (torch.randn(shape, generator=g, device=dev, dtype=torch.float32) * spec.std).to(bf)

        self.layers = []
        for li in range(spec.layers):
            g = torch.Generator(device=dev)
            g.manual_seed(seed * 1000003 + li)
            wq = normal(g, (L.q_dim, L.hidden))
            wk = normal(g, (L.kv_dim, L.hidden))
            wv = normal(g, (L.kv_dim, L.hidden))
            wqkv = torch.cat([wq[q0:q1], wk[k0:k1], wv[k0:k1]]).contiguous()
            del wq, wk, wv
            wo = normal(g, (L.hidden, L.q_dim))[:, q0:q1].contiguous()
            wg = normal(g, (L.intermediate, L.hidden))
            wu = normal(g, (L.intermediate, L.hidden))
            if inter % 64 == 0:
                # gate and up rows interleaved in blocks of 64, the layout of
                # the fused gate|up projection + SwiGLU (mslim_cuda_gemv_swiglu)
                wgu = _att.interleave_gate_up(wg[i0:i0 + inter], wu[i0:i0 + inter])
            else:
                wgu = torch.cat([wg[i0:i0 + inter], wu[i0:i0 + inter]]).contiguous()
            del wg, wu
            wd = normal(g, (L.hidden, L.intermediate))[:, i0:i0 + inter].contiguous()
            ones = torch.full((L.hidden,), 1.0, dtype=bf, device=dev)
            self.layers.append({"in_norm": ones, "post_norm": ones.clone(), "wqkv": wqkv, "wo": wo,
                                "wgu": wgu, "wd": wd})
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 1000003 + 999983)
        self.embedding = normal(g, (spec.vocab, L.hidden))   # tied: lm_head = embedding
        # the lm_head is split by vocabulary rows; the embedding lookup keeps
        # the whole table (any token id can come in)
        per = (spec.vocab + tp_world - 1) // tp_world
        self.vocab_lo = min(tp_rank * per, spec.vocab)
        self.vocab_hi = min(self.vocab_lo + per, spec.vocab)
        self.lm_head = self.embedding[self.vocab_lo:self.vocab_hi]
        self.final_norm = torch.full((L.hidden,), 1.0, dtype=bf, device=dev)
        self.inter = inter
        self.gu_interleaved = inter % 64 == 0
        # K/V of this rank's heads, per layer
        if kv_mode == "dense":
            self.k_cache = [torch.zeros((batch, capacity, self.kvh, D), dtype=bf, device=dev)
                            for _ in range(spec.layers)]
            self.v_cache = [torch.zeros_like(c) for c in self.k_cache]
            reach = capacity
        else:
            self.page_tokens = page_tokens
            self.max_pages = (capacity + page_tokens - 1) // page_tokens
            n_pages = batch * self.max_pages
            # session s owns pages s*max_pages.. in a fixed random physical order
            perm = torch.randperm(n_pages, generator=torch.Generator().manual_seed(seed), dtype=torch.int64)
            self.page_table = perm.to(torch.int32).reshape(batch, self.max_pages).to(dev)
            self.n_pages = n_pages
            self.k_pool = [torch.zeros((n_pages, self.kvh, page_tokens, D), dtype=bf, device=dev)
                           for _ in range(spec.layers)]
            self.v_pool = [torch.zeros_like(p) for p in self.k_pool]
            reach = self.max_pages * page_tokens
        ws = _att.decode_workspace_bytes(self.geometry, batch, reach)
        self.workspace = torch.zeros(max(ws, 16), dtype=torch.uint8, device=dev)
        self.lengths = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.host_length = 0  # every session's token count, mirrored on the host
        self.profile = None   # a SectionTimer splits the device time by kind of step
        # decode-step reductions over NVLink peer memory (fused with the
        # residual add and RMSNorm); prefill reduces through NCCL
        self.comm = None
        if tp_world > 1:
            from .tp import TpComm
            self.comm = TpComm(tp_world, tp_rank, batch, L.hidden, group)

    # ------------------------------------------------------------ pieces --
    def _sec(self, kind, op=None, nbytes=0, kernel=None, link="hbm"):
        if self.profile is None:
            return _NO_SECTION
        return self.profile(kind, op, nbytes, kernel, link)

    def _row_bytes(self, rows, width, passes):
        """bf16 bytes of `passes` reads or writes of a [rows][width] tensor."""
        return 2 * rows * width * passes

    def _all_reduce(self, x):
        if self.world > 1:
            import torch.distributed as dist
            with self._sec("collective"):
                dist.all_reduce(x, op=dist.ReduceOp.SUM, group=self.group)

    def _norm(self, x, w):
        out = self.torch.empty_like(x)
        H = self.spec.layer.hidden
        with self._sec("elementwise", "rmsnorm", self._row_bytes(x.shape[0], H, 2) + 2 * H, "mslim_rmsnorm"):
            _att.rmsnorm(x, w, out, x.shape[0], self.spec.layer.hidden, self.spec.layer.eps)
        return out

    def _gemm(self, x, w, out=None, op="gemm"):
        """x @ w^T: the decode step's few rows (decode_gemm="own") through
        mslim_cuda_gemv, the tcgen05 weight-streaming projection; prefill rows
        (and decode_gemm="cublas") through cuBLAS."""
        t = self.torch
        rows, (n, k) = x.shape[0], w.shape
        own = self.decode_gemm == "own" and rows <= 16 and k % 8 == 0
        nbytes = 2 * (n * k + rows * k + rows * n)
        with self._sec("gemm", op, nbytes, "mslim_gemv_tc" if own else "cuBLAS GEMM"):
            if own:
                y = out if out is not None else t.empty((rows, n), dtype=x.dtype, device=self.device)
                _att.gemv(x.contiguous(), w, y, rows, n, k)
                return y
            if out is not None:
                return t.matmul(x, w.t(), out=out)
            return t.matmul(x, w.t())

    def _qkv_split(self, qkv):
        D = self.spec.layer.head_dim
        nq, nk = self.qh * D, self.kvh * D
        with self._sec("elementwise"):
            return (qkv[:, :nq].contiguous(), qkv[:, nq:nq + nk].contiguous(),
                    qkv[:, nq + nk:].contiguous())

    def _residual_norm(self, x, delta, w):
        """x = bf16(x + delta) in place; returns RMSNorm(x, w)."""
        out = self.torch.empty_like(x)
        H = self.spec.layer.hidden
        with self._sec("elementwise", "residual + RMSNorm", self._row_bytes(x.shape[0], H, 4) + 2 * H,
                       "mslim_rmsnorm<residual>"):
            _att.residual_rmsnorm(x, delta, w, out, x.shape[0], self.spec.layer.hidden, self.spec.layer.eps)
        return out

    def _reduce_residual_norm(self, inp, w_proj, x, w_norm, reduce: bool, fused: bool, op="gemm"):
        """x += (sum over ranks of) inp @ w_proj^T; returns RMSNorm(x, w_norm).
        fused: the GEMM writes this rank's partial into the communicator slot
        and one kernel reduces over NVLink, adds and normalises (decode);
        otherwise NCCL all-reduce then the fused residual + RMSNorm."""
        rows = x.shape[0]
        if reduce and fused and self.comm is not None:
            slot = self.comm.next_slot()
            self._gemm(inp, w_proj, out=self.comm.slot(slot, rows), op=op)
            out = self.torch.empty_like(x)
            H = self.spec.layer.hidden
            # the bytes that cross NVLink into this rank: every peer's partial row
            with self._sec("collective", "NVLink reduce + residual + RMSNorm",
                           self._row_bytes(rows, H, self.world - 1), "mslim_tp_allreduce_rmsnorm", "nvlink"):
                self.comm.allreduce_rmsnorm(slot, x, w_norm, out, rows, self.spec.layer.eps)
            return out
        y = self._gemm(inp, w_proj, op=op)
        if reduce:
            self._all_reduce(y)
        return self._residual_norm(x, y, w_norm)

    def _after_attention(self, li, x, attn, fused: bool = False):
        """o-projection (+ reduction), residual, MLP (+ reduction when
        sharded), residual; returns the next layer's normalised input (the
        final norm after the last layer)."""
        t = self.torch
        W = self.layers[li]
        n2 = self._reduce_residual_norm(attn.reshape(x.shape[0], -1), W["wo"], x, W["post_norm"], True, fused,
                                        op="o projection")
        rows, H = x.shape[0], self.spec.layer.hidden
        act = t.empty((rows, self.inter), dtype=x.dtype, device=self.device)
        if self.gu_interleaved and self.decode_gemm == "own" and rows <= 16:
            # one launch: the projection's epilogue applies SwiGLU
            nbytes = 2 * (2 * self.inter * H + rows * H + rows * self.inter)
            with self._sec("gemm", "gate|up projection + SwiGLU", nbytes, "mslim_gemv_tc<swiglu>"):
                _att.gemv_swiglu(n2, W["wgu"], act, rows, self.inter, H)
        else:
            gu = self._gemm(n2, W["wgu"], op="gate|up projection")
            with self._sec("elementwise", "SwiGLU", self._row_bytes(rows, self.inter, 3), "mslim_swiglu_rows"):
                if self.gu_interleaved:
                    # every 128-wide block of a row is one [gate 64 | up 64] pair
                    _att.swiglu_rows(gu, act, rows * self.inter // 64, 64)
                else:
                    _att.swiglu_rows(gu, act, rows, self.inter)
        nxt = self.layers[li + 1]["in_norm"] if li + 1 < len(self.layers) else self.final_norm
        return self._reduce_residual_norm(act, W["wd"], x, nxt, self.mlp == "sharded", fused, op="down projection")

    def _lm_head_argmax(self, n_final):
        """n_final: final-normed bf16 [batch][hidden] -> (int32 ids, bf16 logits
        of this rank's vocabulary slice).  With several ranks each takes the
        argmax of its slice and one all-gather of (total-order key, index)
        pairs picks the winner; equal keys go to the larger index, so the
        CPU path's tie rule (last maximal index) holds across slices."""
        t = self.torch
        B = n_final.shape[0]
        logits = self._gemm(n_final, self.lm_head, op="lm_head")
        ids = t.empty(B, dtype=t.int32, device=self.device)
        with self._sec("elementwise", "argmax", self._row_bytes(B, self.vocab_hi - self.vocab_lo, 1),
                       "mslim_argmax"):
            _att.argmax(logits, B, self.vocab_hi - self.vocab_lo, ids, ties_to_last=True)
        if self.world == 1:
            return ids, logits
        import torch.distributed as dist
        with self._sec("elementwise", "argmax shard key", 0, "torch elementwise"):
            bits = logits.gather(1, ids.long().view(B, 1)).view(t.int16).view(B)
            mine = shard_argmax_key(t, bits, ids, self.vocab_lo)
            every = t.empty((self.world, B), dtype=t.int64, device=self.device)
        with self._sec("collective", "argmax all-gather", 8 * B * (self.world - 1), "NCCL all_gather", "nvlink"):
            dist.all_gather_into_tensor(every, mine, group=self.group)
        with self._sec("elementwise", "argmax shard key", 0, "torch elementwise"):
            best = pick_shard_argmax(t, every)
        return best, logits

    # ----------------------------------------------------------- prefill --
    def prefill(self, ids):
        """ids: int64 [batch][S] prompt tokens (positions 0..S-1 of every
        session).  Returns the greedy next token per session (and logits)."""
        t, L = self.torch, self.spec.layer
        B, S = ids.shape
        D = L.head_dim
        if S > self.capacity:
            raise ValueError("prompt longer than the K/V capacity")
        with self._sec("elementwise"):
            x = self.embedding.index_select(0, ids.reshape(-1)).contiguous()   # [B*S][hidden]
        n = self._norm(x, self.layers[0]["in_norm"])
        for li, W in enumerate(self.layers):
            q, k, v = self._qkv_split(self._gemm(n, W["wqkv"]))
            q_r = t.empty_like(q)
            k_r = t.empty_like(k)
            attn = t.empty_like(q)
            for b in range(B):
                rows = slice(b * S, (b + 1) * S)
                with self._sec("elementwise"):
                    _att.rope(q[rows], q_r[rows], S, self.qh, D, 0, self.rope_cfg)
                    _att.rope(k[rows], k_r[rows], S, self.kvh, D, 0, self.rope_cfg)
                    if self.kv_mode == "dense":
                        self.k_cache[li][b, :S] = k_r[rows].view(S, self.kvh, D)
                        self.v_cache[li][b, :S] = v[rows].view(S, self.kvh, D)
                    else:
                        q_tmp = t.empty((S, self.qh * D), dtype=q.dtype, device=self.device)
                        _att.rope_append_paged(self.geometry, q[rows], q_tmp, k[rows], v[rows], S, 0,
                                               self.rope_cfg, self.k_pool[li], self.v_pool[li],
                                               self.n_pages, self.page_tokens, self.page_table[b:b + 1],
                                               self.max_pages)
                with self._sec("attention"):
                    _att.prefill_causal(self.geometry, q_r[rows], k_r[rows], v[rows], attn[rows], S, 0)
            n = self._after_attention(li, x, attn)
        self.lengths.fill_(S)
        self.host_length = S
        last = n.view(B, S, L.hidden)[:, S - 1].contiguous()
        return self._lm_head_argmax(last)

    # ------------------------------------------------------------ decode --
    def decode_step(self, tokens):
        """tokens: int32 [batch] (this step's input token per session, at
        position lengths[b]).  Returns (next tokens, logits)."""
        t = self.torch
        B = tokens.shape[0]
        D = self.spec.layer.head_dim
        H = self.spec.layer.hidden
        with self._sec("elementwise", "embedding gather", self._row_bytes(B, H, 2), "torch index_select"):
            x = self.embedding.index_select(0, tokens.long()).contiguous()    # [B][hidden]
            pos = self.lengths
            seq = pos + 1
        # algorithmic bytes of this step's rope + append and attention (every
        # session holds host_length tokens before the step)
        rope_bytes = self._row_bytes(B, (2 * self.qh + 4 * self.kvh) * D, 1)
        ctx = self.host_length + 1
        attn_bytes = self._row_bytes(B * ctx, self.kvh * D, 2) + self._row_bytes(B, self.qh * D, 2)
        paged = self.kv_mode != "dense"
        rope_name = "mslim_rope_append_paged" if paged else "mslim_rope_append_dense"
        attn_name = ("mslim_decode_persist" if _att.get_decode_schedule() == _att.DECODE_PERSISTENT
                     else "mslim_decode_split + mslim_decode_merge_row")
        # fuse_qkv: one launch for the q|k|v projection, RoPE and the K/V
        # append (own projection, head_dim 128: a head per tile).  Off by
        # default: in graph-replayed steps the separate append kernel overlaps
        # the projection's tail (programmatic dependent launch) and measured
        # ~1.7 % faster per step; the fused form saves a launch when steps are
        # issued eagerly.
        fused_qkv = self.fuse_qkv and self.decode_gemm == "own" and D == 128 and B <= 16 and H % 8 == 0
        qkv_bytes = 2 * ((self.qh + 2 * self.kvh) * D * H + B * H) + rope_bytes // 2
        n = self._norm(x, self.layers[0]["in_norm"])
        for li, W in enumerate(self.layers):
            q_r = t.empty((B, self.qh * D), dtype=x.dtype, device=self.device)
            attn = t.empty_like(q_r)
            if fused_qkv:
                with self._sec("gemm", "q|k|v projection + RoPE + K/V append", qkv_bytes,
                               "mslim_gemv_tc<rope_append>"):
                    if self.kv_mode == "dense":
                        _att.gemv_qkv_rope_append_dense(self.geometry, n, W["wqkv"], H, pos, B, self.rope_cfg, q_r,
                                                        self.k_cache[li], self.v_cache[li], self.capacity)
                    else:
                        _att.gemv_qkv_rope_append_paged(self.geometry, n, W["wqkv"], H, pos, B, self.rope_cfg, q_r,
                                                        self.k_pool[li], self.v_pool[li], self.n_pages,
                                                        self.page_tokens, self.page_table, self.max_pages)
            else:
                qkv = self._gemm(n, W["wqkv"], op="q|k|v projection")
            if self.kv_mode == "dense":
                if not fused_qkv:
                    with self._sec("elementwise", "RoPE + K/V append", rope_bytes, rope_name):
                        _att.rope_append_decode_dense_qkv(self.geometry, qkv, q_r, pos, B, self.rope_cfg,
                                                          self.k_cache[li], self.v_cache[li], self.capacity)
                with self._sec("attention", "decode attention", attn_bytes, attn_name):
                    _att.decode_dense(self.geometry, q_r, self.k_cache[li], self.v_cache[li], seq, B,
                                      self.capacity, self.workspace, attn)
            else:
                if not fused_qkv:
                    with self._sec("elementwise", "RoPE + K/V append", rope_bytes, rope_name):
                        _att.rope_append_decode_paged_qkv(self.geometry, qkv, q_r, pos, B, self.rope_cfg,
                                                          self.k_pool[li], self.v_pool[li], self.n_pages,
                                                          self.page_tokens, self.page_table, self.max_pages)
                with self._sec("attention", "decode attention", attn_bytes, attn_name):
                    _att.decode_paged(self.geometry, q_r, self.k_pool[li], self.v_pool[li], self.n_pages,
                                      self.page_tokens, self.page_table, self.max_pages, seq, B,
                                      self.workspace, attn)
            n = self._after_attention(li, x, attn, fused=True)
        with self._sec("elementwise", "positions", 8 * B, "torch add"):
            self.lengths.add_(1)
        self.host_length += 1
        return self._lm_head_argmax(n)

    # --------------------------------------------------- validation digest --
    def logical_kv_sha256(self, session: int = 0) -> str:
        """The adapters' validation digest of one session's K/V state over
        all layers (GpuLlm::logical_kv_sha256, src/gpu_llm/mod.rs:1981-2023):
        "mslim-dense-kv-state-v1", the session's token count, then per layer K
        and V ordered [kv_heads][tokens][head_dim] (this rank's KV heads).
        Equal for the dense and the ColdStore-exact store when they hold the
        same bf16 K/V."""
        from .digest import LogicalKvHasher, device_tensor_bytes
        t, D = self.torch, self.spec.layer.head_dim
        T = int(self.lengths[session].item())
        hasher = LogicalKvHasher(T)
        k = t.empty((self.kvh, T, D), dtype=t.bfloat16, device=self.device)
        v = t.empty_like(k)
        for li in range(self.spec.layers):
            if self.kv_mode == "dense":
                _att.kv_canonical_dense(self.k_cache[li][session], self.kvh, D, T, k)
                _att.kv_canonical_dense(self.v_cache[li][session], self.kvh, D, T, v)
            else:
                row = self.page_table[session]
                _att.kv_canonical_paged(self.k_pool[li], self.n_pages, self.kvh, self.page_tokens, D, row,
                                        self.max_pages, T, k)
                _att.kv_canonical_paged(self.v_pool[li], self.n_pages, self.kvh, self.page_tokens, D, row,
                                        self.max_pages, T, v)
            hasher.add(device_tensor_bytes(t, k), device_tensor_bytes(t, v))
        if _att.device_status(self.device.index or 0) != 0:
            raise _att.ShapeMismatch("a page id outside the pool while reading the K/V state")
        return hasher.hexdigest()

    # ------------------------------------------------------- graph decode --
    def capture_decode(self):
        """Captures one whole decode step (every layer, the all-reduces, the
        lm_head and the argmax) into a CUDA graph.  decode_step_graphed then
        replays it: the host issues one launch per step instead of ~20 per
        layer, and positions advance on the device (lengths += 1 is part of
        the graph).  Call after at least one eager decode step."""
        t = self.torch
        self.g_tokens = t.zeros(self.batch, dtype=t.int32, device=self.device)
        saved = self.lengths.clone()
        saved_host = self.host_length
        self.graph = t.cuda.CUDAGraph()
        side = t.cuda.Stream()
        side.wait_stream(t.cuda.current_stream())
        with t.cuda.graph(self.graph, stream=side):
            self.g_out, self.g_logits = self.decode_step(self.g_tokens)
        t.cuda.current_stream().wait_stream(side)
        # capturing ran nothing; keep the lengths the caller had
        self.lengths.copy_(saved)
        self.host_length = saved_host

    def decode_step_graphed(self, tokens):
        self.g_tokens.copy_(tokens)
        self.graph.replay()
        self.host_length += 1
        return self.g_out, self.g_logits

    def release_graph(self):
        """Drops the captured graph (before the process group goes away)."""
        self.graph = None
        self.g_out = self.g_logits = None

    def close(self):
        """Releases the graph and the communicator's peer mappings (call on
        every rank, before the process group is destroyed)."""
        self.release_graph()
        if self.comm is not None:
            if self.world > 1:
                import torch.distributed as dist
                self.torch.cuda.synchronize()
                dist.barrier(group=self.group)
            self.comm.close()
            self.comm = None

