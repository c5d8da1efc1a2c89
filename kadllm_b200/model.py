"""Native BF16 execution of the hybrid Qwen3.5 stack for GRBeam.

``HybridModel`` holds the weights packed for this pipeline (one input GEMM per
token mixer and per MLP) and runs

* ``prefill(ids)``: the prompt through every layer (conv + chunked gated delta
  rule for GDN layers, causal flash attention for full-attention layers),
  producing the first-token logits and the immutable, request-sized prefix
  (conv state, recurrent state, K/V) exactly where the reference keeps them
  (``Qwen35GRBeamAdapter.prefill``, ``src/kadllm/adapters/qwen3_5.py:106-133``);
* ``decode(history, state)``: suffix replay of every beam from the shared
  prefix (``Qwen35GRBeamAdapter.decode``, ``src/kadllm/adapters/qwen3_5.py:204-235``)
  through the fused GDN mixer and the shared-prefix attention kernels.

Token mixers, norms, attention, selection and every projection are
hand-written sm_100a kernels (``csrc/``): the projections and the LM head run
on the library's tcgen05 GEMM (``kadllm_gemm``), with the MLP's SiLU-mul and
the residual updates fused into its epilogue.  Everything stays on the GPU;
there is no CPU path.
"""

from __future__ import annotations

import threading

from dataclasses import dataclass

import torch

from . import _lib
from .config import LINEAR, HybridConfig

BF16 = torch.bfloat16

# epilogues of kadllm_gemm
GEMM_STORE, GEMM_SILU_MUL, GEMM_ADD = 0, 1, 2
GATE_UP_BLOCK = 128  # rows per gate / up block of the interleaved MLP input weight


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """gate, up [I, H] -> [2 I', H]: 128-row blocks [gate block j | up block j], I' = I
    rounded up to a multiple of 128 (zero rows), the layout of kadllm_gemm's SiLU-mul
    epilogue (one 256-column tile of the product holds matching gate and up columns)."""
    inter, hidden = gate.shape
    padded = -(-inter // GATE_UP_BLOCK) * GATE_UP_BLOCK
    if padded != inter:
        gate = torch.cat([gate, gate.new_zeros(padded - inter, hidden)])
        up = torch.cat([up, up.new_zeros(padded - inter, hidden)])
    n = padded // GATE_UP_BLOCK
    return torch.stack([gate.reshape(n, GATE_UP_BLOCK, hidden), up.reshape(n, GATE_UP_BLOCK, hidden)], 1) \
        .reshape(2 * padded, hidden).contiguous()


@dataclass
class GDNLayer:
    w_in: torch.Tensor      # [conv_dim + value_dim + 2*HV, H]: qkv | z | b | a
    w_out: torch.Tensor     # [H, value_dim]
    conv_w: torch.Tensor    # [conv_dim, 4]
    a_log: torch.Tensor     # [HV] f32
    dt_bias: torch.Tensor   # [HV] f32
    norm_w: torch.Tensor    # [V] f32


@dataclass
class AttnLayer:
    w_in: torch.Tensor      # [(2*Hq + 2*HK) * D, H]: (q|gate) per head | k | v
    w_o: torch.Tensor       # [H, Hq*D]
    q_norm: torch.Tensor    # [D] f32
    k_norm: torch.Tensor    # [D] f32


@dataclass
class Layer:
    kind: str
    mixer: GDNLayer | AttnLayer
    input_ln: torch.Tensor  # [H] f32
    post_ln: torch.Tensor   # [H] f32
    w_gu: torch.Tensor      # [2*I', H]: gate / up interleaved in 128-row blocks (interleave_gate_up)
    w_down: torch.Tensor    # [H, I]
    inter: int              # I, the MLP width of this layer


TILED_HEAD_DIM = 256  # head dim of the tensor-core attention kernels


@dataclass(frozen=True)
class HybridPrefix:
    """Immutable request-sized prefix (``Qwen35Prefix``, ``src/kadllm/adapters/qwen3_5.py:21-26``).

    ``layers[i]`` is (conv_state [B, conv_dim, 4], recurrent_state [B, HV, K, V])
    for GDN layers and (K, V) as [B, L, HK, D] views of [B, HK, L, D] caches
    for attention layers -- the reference's layouts and BF16 dtypes.
    """

    length: int  # the prefix length (the longest one for packed prompts)
    batch: int
    owner: object
    layers: tuple
    # attention layers: (K tiles, V tiles, blocks per head) for the tensor-core kernels, else None
    tiles: tuple = ()
    # packed prompts of their own lengths (``prefill_varlen``): device int32 offsets [B + 1]
    # and the host lengths; attention layers then hold packed [rows, HK, D] K / V
    cu: torch.Tensor | None = None
    lengths: tuple = ()


class HybridModel:
    def __init__(self, cfg: HybridConfig, weights: dict[str, torch.Tensor], device=None):
        cfg.validate()
        self.cfg = cfg
        dev = torch.device(device) if device is not None else next(iter(weights.values())).device
        if dev.type != "cuda":
            raise RuntimeError("kadllm_b200 runs on CUDA devices only")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        _lib.lib()  # fail loudly now if the CUDA library is missing

        def bf(name):
            return weights[name].to(device=dev, dtype=BF16).contiguous()

        def f32(name):
            return weights[name].to(device=dev, dtype=torch.float32).contiguous()

        self.embed = bf("embed_tokens.weight")
        self.lm_head = bf("lm_head.weight") if "lm_head.weight" in weights else self.embed
        self.final_norm = f32("norm.weight")
        self.layers: list[Layer] = []
        for i, kind in enumerate(cfg.layer_types):
            p = f"layers.{i}."
            if kind == LINEAR:
                q = p + "linear_attn."
                w_in = torch.cat([bf(q + "in_proj_qkv.weight"), bf(q + "in_proj_z.weight"),
                                  bf(q + "in_proj_b.weight"), bf(q + "in_proj_a.weight")])
                pad = (-w_in.shape[0]) % 8  # 16-byte projection rows for vector loads
                if pad:
                    w_in = torch.cat([w_in, w_in.new_zeros(pad, w_in.shape[1])])
                mixer = GDNLayer(
                    w_in=w_in.contiguous(),
                    w_out=bf(q + "out_proj.weight"),
                    conv_w=bf(q + "conv1d.weight").reshape(cfg.conv_dim, -1).contiguous(),
                    a_log=f32(q + "A_log"), dt_bias=f32(q + "dt_bias"), norm_w=f32(q + "norm.weight"))
            else:
                q = p + "self_attn."
                mixer = AttnLayer(
                    w_in=torch.cat([bf(q + "q_proj.weight"), bf(q + "k_proj.weight"),
                                    bf(q + "v_proj.weight")]).contiguous(),
                    w_o=bf(q + "o_proj.weight"), q_norm=f32(q + "q_norm.weight"),
                    k_norm=f32(q + "k_norm.weight"))
            self.layers.append(Layer(
                kind=kind, mixer=mixer, input_ln=f32(p + "input_layernorm.weight"),
                post_ln=f32(p + "post_attention_layernorm.weight"),
                w_gu=interleave_gate_up(bf(p + "mlp.gate_proj.weight"), bf(p + "mlp.up_proj.weight")),
                w_down=bf(p + "mlp.down_proj.weight"), inter=int(weights[p + "mlp.gate_proj.weight"].shape[0])))
        self._rope_len = 0
        self._cos = self._sin = None
        self._rope_lock = threading.Lock()
        self._rope_retired = []  # outgrown tables stay alive: kernels on other streams may still read them
        self.owner = object()
        # device status word of the tensor-core kernels (bit 0: a bounded wait timed out)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)

    @property
    def step_reuse(self) -> bool:
        """Whether a two-token decode can continue from the one-token step's cache (the
        continuing GDN mixer takes head dims 64 / 128 with K == V)."""
        c = self.cfg
        return c.linear_key_head_dim == c.linear_value_head_dim and c.linear_key_head_dim in (64, 128)

    def fused_select(self, batch: int, width: int) -> bool:
        """Whether a decode step of batch x width rows can run the LM head with the
        selection's chunk statistics in its epilogue (vocabulary a multiple of 8, at most
        393216 columns)."""
        V = self.lm_head.shape[0]
        return V % 8 == 0 and V <= 393216 and batch * width >= 1

    def check(self) -> None:
        """Raise if a tensor-core kernel reported a timed-out wait (synchronises)."""
        st = int(self.status.item())
        if st:
            raise RuntimeError(f"kadllm_b200: device status {st:#x} (a tensor-core pipeline wait timed out)")

    def _tile_kv(self, kc, vc, strides):
        """[B, HK, L, D] caches -> the tiled K / V images the tensor-core attention stages."""
        B, hk, L, D = kc.shape
        nbytes = _lib.lib().kadllm_kv_tile_bytes(B, hk, L, D)
        if nbytes <= 0:
            return None
        kt = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        vt = torch.empty_like(kt)
        s = self._stream()
        _lib.call("kadllm_kv_tile", kc.data_ptr(), *strides, B, hk, L, D, kt.data_ptr(), nbytes, s)
        _lib.call("kadllm_kv_tile", vc.data_ptr(), *strides, B, hk, L, D, vt.data_ptr(), nbytes, s)
        return kt, vt, -(-L // 64)

    # ------------------------------------------------------------------ helpers
    def _stream(self):
        return _lib.stream(self.device)

    def _rope(self, n: int):
        """cos/sin tables [n, rotary_dim] in BF16, computed like
        ``Qwen3_5TextRotaryEmbedding`` (fp32 inv_freq x position, cos/sin, cast)."""
        with self._rope_lock:
            if n > self._rope_len:
                n = max(n, 2 * self._rope_len, 4096)
                rd = self.cfg.rotary_dim
                inv = 1.0 / (self.cfg.rope_theta ** (torch.arange(0, rd, 2, dtype=torch.int64, device=self.device)
                                                     .float() / rd))
                pos = torch.arange(n, device=self.device, dtype=torch.float32)
                freqs = pos[:, None] * inv[None, :]
                emb = torch.cat([freqs, freqs], -1)
                cos, sin = emb.cos().to(BF16).contiguous(), emb.sin().to(BF16).contiguous()
                torch.cuda.current_stream(self.device).synchronize()  # complete before any stream reads it
                if self._cos is not None:
                    self._rope_retired.append((self._cos, self._sin))
                self._cos, self._sin, self._rope_len = cos, sin, n
            return self._cos, self._sin

    def _embed(self, ids: torch.Tensor):
        rows = ids.numel()
        H = self.cfg.hidden_size
        x = torch.empty(rows, H, dtype=BF16, device=self.device)
        normed = torch.empty_like(x)
        _lib.call("kadllm_embed_rmsnorm", ids.data_ptr(), self.embed.data_ptr(), self.cfg.vocab_size,
                  self.layers[0].input_ln.data_ptr(), self.cfg.rms_norm_eps, x.data_ptr(), normed.data_ptr(),
                  rows, H, self._stream())
        return x, normed

    def _add_norm(self, x, delta, weight, normed, rows=None, step=1, offset=0):
        rows = x.shape[0] if rows is None else rows
        _lib.call("kadllm_add_rmsnorm", x.data_ptr(), _lib.ptr(delta), 0 if delta is None else delta.stride(0),
                  weight.data_ptr(), self.cfg.rms_norm_eps, normed.data_ptr(), rows, step, offset,
                  self.cfg.hidden_size, self._stream())

    def _gemm(self, a: torch.Tensor, w: torch.Tensor, *, resid: torch.Tensor | None = None,
              silu_inter: int | None = None) -> torch.Tensor:
        """a [M, K] . w[N, K]^T on the tcgen05 GEMM.  ``resid``: x += a . w^T in place
        (returns x); ``silu_inter``: w is an interleave_gate_up weight, returns the
        [M, silu_inter] SiLU-mul activation; otherwise a new [M, N] product."""
        M, K = a.shape
        N = w.shape[0]
        if silu_inter is not None:
            epi, n_out = GEMM_SILU_MUL, silu_inter
            out = torch.empty(M, n_out, dtype=BF16, device=self.device)
        elif resid is not None:
            epi, n_out, out = GEMM_ADD, N, resid
        else:
            epi, n_out = GEMM_STORE, N
            out = torch.empty(M, N, dtype=BF16, device=self.device)
        _lib.call("kadllm_gemm", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(), out.stride(0),
                  _lib.ptr(resid), 0 if resid is None else resid.stride(0), M, N, K, n_out, epi,
                  self.status.data_ptr(), self._stream())
        return out

    def _mixer_records_ok(self) -> bool:
        """The staged decode mixer keeps first-step records (head dims 64 / 128, K == V)."""
        c = self.cfg
        return c.linear_key_head_dim == c.linear_value_head_dim and c.linear_key_head_dim in (64, 128)

    def _mlp(self, layer: Layer, normed, x):
        """x += down(silu(gate(normed)) * up(normed)): two GEMMs, the activation and the
        residual update in their epilogues (per layer width: WideTuning-merged layers are wider)."""
        act = self._gemm(normed, layer.w_gu, silu_inter=layer.inter)
        self._gemm(act, layer.w_down, resid=x)

    def _qk_rope(self, P, rows, pos_base, rows_per_seq, q_out, k_out, k_strides, v_out, v_strides, mixer,
                 pos_of_row=None, max_pos=None, q_row_stride=None):
        c = self.cfg
        cos, sin = self._rope((pos_base + rows_per_seq if max_pos is None else max_pos) + 1)
        _lib.call("kadllm_qk_norm_rope", P.data_ptr(), P.stride(0), c.num_attention_heads, c.num_key_value_heads,
                  c.head_dim, mixer.q_norm.data_ptr(), mixer.k_norm.data_ptr(), c.rms_norm_eps, cos.data_ptr(),
                  sin.data_ptr(), c.rotary_dim, _lib.ptr(pos_of_row), pos_base, rows_per_seq, q_out.data_ptr(),
                  q_row_stride or c.num_attention_heads * c.head_dim, c.head_dim, k_out.data_ptr(), *k_strides,
                  v_out.data_ptr(), *v_strides, rows, self._stream())

    def _gather_rows(self, src: torch.Tensor, parent: torch.Tensor, width: int, prev_width: int,
                     dst: torch.Tensor, dst_row_stride: int):
        """dst row i <- src row (i // width) * prev_width + parent[i] (rows of ``src`` [B*prev_width, n],
        contiguous; ``dst`` a view whose rows are ``dst_row_stride`` elements apart)."""
        n = src.shape[1]
        esz = src.element_size()
        _lib.call("kadllm_gather_rows", src.data_ptr(), n * esz, parent.data_ptr(), width, prev_width,
                  parent.numel(), n * esz, dst.data_ptr(), dst_row_stride * esz, self._stream())

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def prefill(self, ids: torch.Tensor, head: torch.Tensor | None = None, taps: list | None = None):
        """ids [B, L] -> (logits [B, V] bf16, HybridPrefix).  ``head`` [V', H] replaces
        the LM head (a SID-only head: logits over its rows only).  ``taps``, when given,
        receives the hidden state of every request's last prompt position after each
        decoder layer ([B, H] fp32 copies, for layer-by-layer parity checks)."""
        c = self.cfg
        B, L = ids.shape
        ids = ids.to(device=self.device, dtype=torch.int64).contiguous()
        R = B * L
        x, normed = self._embed(ids.reshape(-1))
        s = self._stream()
        prefix = []
        tiles = []
        hk, D, hq = c.num_key_value_heads, c.head_dim, c.num_attention_heads
        ws = None  # GDN prefill workspace (chunk blocks), shared by the GDN layers
        for i, layer in enumerate(self.layers):
            m = layer.mixer
            P = self._gemm(normed, m.w_in)
            if layer.kind == LINEAR:
                conv_state = torch.empty(B, c.conv_dim, 4, dtype=BF16, device=self.device)
                out = torch.empty(R, c.value_dim, dtype=BF16, device=self.device)
                rec = torch.empty(B, c.linear_num_value_heads, c.linear_key_head_dim, c.linear_value_head_dim,
                                  dtype=BF16, device=self.device)
                if ws is None:
                    ws = torch.empty(_lib.lib().kadllm_gdn_prefill_workspace(
                        B, L, c.linear_num_value_heads, c.linear_key_head_dim, c.linear_value_head_dim),
                        dtype=torch.uint8, device=self.device)
                _lib.call("kadllm_gdn_prefill_split", P.data_ptr(), P.stride(0), m.conv_w.data_ptr(),
                          conv_state.data_ptr(), m.a_log.data_ptr(), m.dt_bias.data_ptr(), m.norm_w.data_ptr(),
                          c.rms_norm_eps, out.data_ptr(), out.stride(0), rec.data_ptr(), ws.data_ptr(), ws.numel(),
                          B, L, c.linear_num_key_heads, c.linear_num_value_heads, c.linear_key_head_dim,
                          c.linear_value_head_dim, s)
                w_post = m.w_out
                prefix.append((conv_state, rec))
                tiles.append(None)
            else:
                q = torch.empty(R, hq, D, dtype=BF16, device=self.device)
                kc = torch.empty(B, hk, L, D, dtype=BF16, device=self.device)
                vc = torch.empty_like(kc)
                cache_strides = (hk * L * D, D, L * D)  # (sequence, position, head)
                self._qk_rope(P, R, 0, L, q, kc, cache_strides, vc, cache_strides, m)
                out = torch.empty(R, hq * D, dtype=BF16, device=self.device)
                gate = P[:, D:]  # gate of head h at column h*2D + D
                tile = self._tile_kv(kc, vc, cache_strides) if D == TILED_HEAD_DIM else None
                if tile is not None:  # tensor-core kernel over the tiled prefix
                    kt, vt, nblk = tile
                    _lib.call("kadllm_attention_tiled", q.data_ptr(), hq * D, 0, D, kt.data_ptr(), vt.data_ptr(),
                              nblk, None, 0, 0, 0, None, 0, 0, 0, gate.data_ptr(), P.stride(0), 0, 2 * D,
                              out.data_ptr(), out.stride(0), 0, D, self.status.data_ptr(), B, 1, 1, 0, hq, hk, L, D,
                              D ** -0.5, 1, s)
                else:
                    # cache [B, HK, L, D]: strides passed as (request, position, head)
                    _lib.call("kadllm_causal_attention", q.data_ptr(), hq * D, D, kc.data_ptr(), kc.stride(0),
                              kc.stride(2), kc.stride(1), vc.data_ptr(), vc.stride(0), vc.stride(2), vc.stride(1),
                              gate.data_ptr(), P.stride(0), 2 * D, out.data_ptr(),
                              out.stride(0), D, B, L, hq, hk, D, D ** -0.5, s)
                w_post = m.w_o
                prefix.append((kc.transpose(1, 2), vc.transpose(1, 2)))
                tiles.append(tile)
            if i + 1 < len(self.layers):
                self._post_mixer(layer, out, w_post, x, normed, self.layers[i + 1].input_ln)
                if taps is not None:
                    taps.append(x.view(B, L, -1)[:, -1].float().clone())
        last_rows = torch.arange(B, device=self.device) * L + (L - 1)
        last = self._finish_last_rows(layer, out, w_post, x, last_rows, taps)
        logits = self._gemm(last, self.lm_head if head is None else head)
        return logits, HybridPrefix(L, B, self.owner, tuple(prefix), tuple(tiles))

    def _post_mixer(self, layer: Layer, out, w_post, x, normed, next_ln):
        """x += out . w_post^T; x += MLP(RMSNorm(x)); normed = the next layer's RMSNorm(x)."""
        self._gemm(out, w_post, resid=x)
        self._add_norm(x, None, layer.post_ln, normed)
        self._mlp(layer, normed, x)
        self._add_norm(x, None, next_ln, normed)

    def _finish_last_rows(self, layer: Layer, out, w_post, x, last_rows, taps=None):
        """The last layer after its mixer, for the rows the logits read only (each
        request's last prompt position): the mixer ran over every row for the prefix
        state; its output projection, MLP and the final norm need only these rows.
        Returns the final-norm hidden [len(last_rows), H]."""
        n = last_rows.numel()
        xl = x.index_select(0, last_rows)
        self._gemm(out.index_select(0, last_rows), w_post, resid=xl)
        normed = torch.empty_like(xl)
        self._add_norm(xl, None, layer.post_ln, normed)
        self._mlp(layer, normed, xl)
        if taps is not None:
            taps.append(xl.float().clone())
        last = torch.empty(n, self.cfg.hidden_size, dtype=BF16, device=self.device)
        self._add_norm(xl, None, self.final_norm, last)
        return last

    @torch.no_grad()
    def prefill_varlen(self, prompts, head: torch.Tensor | None = None):
        """Prompts of their own lengths, packed into one batch: ``prompts`` is a list of
        1-D token tensors -> (logits [B, V] bf16, HybridPrefix with ``cu`` / ``lengths``).

        Every kernel sees the packed rows with per-request offsets (device int32
        ``cu``): the GDN prefill runs each request's own chunk count, the causal
        attention each request's own prefix, RoPE each row's own position; the
        prefix K / V are tiled per request.  Head dim 256 attention and 128-dim
        GDN heads only (the tensor-core paths)."""
        c = self.cfg
        hk, D, hq = c.num_key_value_heads, c.head_dim, c.num_attention_heads
        if D != TILED_HEAD_DIM or (c.linear_key_head_dim, c.linear_value_head_dim) != (128, 128):
            raise NotImplementedError("packed prompts need head_dim 256 attention and 128-dim GDN heads")
        lens = [int(p.numel()) for p in prompts]
        if not lens or min(lens) < 1:
            raise ValueError("prompts must be nonempty")
        B, Lmax = len(lens), max(lens)
        offs = [0]
        for n in lens:
            offs.append(offs[-1] + n)
        R = offs[-1]
        ids = torch.cat([p.reshape(-1) for p in prompts]).to(device=self.device, dtype=torch.int64).contiguous()
        cu = torch.tensor(offs, dtype=torch.int32).to(self.device)
        pos = torch.cat([torch.arange(n, dtype=torch.int64) for n in lens]).to(self.device)  # position of each row
        x, normed = self._embed(ids)
        s = self._stream()
        prefix, tiles = [], []
        ws = None
        for i, layer in enumerate(self.layers):
            m = layer.mixer
            P = self._gemm(normed, m.w_in)
            if layer.kind == LINEAR:
                conv_state = torch.empty(B, c.conv_dim, 4, dtype=BF16, device=self.device)
                out = torch.empty(R, c.value_dim, dtype=BF16, device=self.device)
                rec = torch.empty(B, c.linear_num_value_heads, c.linear_key_head_dim, c.linear_value_head_dim,
                                  dtype=BF16, device=self.device)
                if ws is None:
                    ws = torch.empty(_lib.lib().kadllm_gdn_prefill_workspace(
                        B, Lmax, c.linear_num_value_heads, c.linear_key_head_dim, c.linear_value_head_dim),
                        dtype=torch.uint8, device=self.device)
                _lib.call("kadllm_gdn_prefill_split_varlen", P.data_ptr(), P.stride(0), m.conv_w.data_ptr(),
                          conv_state.data_ptr(), m.a_log.data_ptr(), m.dt_bias.data_ptr(), m.norm_w.data_ptr(),
                          c.rms_norm_eps, out.data_ptr(), out.stride(0), rec.data_ptr(), ws.data_ptr(), ws.numel(),
                          cu.data_ptr(), R, B, Lmax, c.linear_num_key_heads, c.linear_num_value_heads,
                          c.linear_key_head_dim, c.linear_value_head_dim, s)
                w_post = m.w_out
                prefix.append((conv_state, rec))
                tiles.append(None)
            else:
                q = torch.empty(R, hq, D, dtype=BF16, device=self.device)
                kp = torch.empty(R, hk, D, dtype=BF16, device=self.device)  # packed rows
                vp = torch.empty_like(kp)
                packed = (0, hk * D, D)  # (sequence, position, head): one run of rows
                self._qk_rope(P, R, 0, R, q, kp, packed, vp, packed, m, pos_of_row=pos, max_pos=Lmax)
                nbytes = _lib.lib().kadllm_kv_tile_bytes(B, hk, Lmax, D)
                kt = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
                vt = torch.empty_like(kt)
                _lib.call("kadllm_kv_tile_varlen", kp.data_ptr(), hk * D, D, cu.data_ptr(), B, hk, Lmax, D,
                          kt.data_ptr(), nbytes, s)
                _lib.call("kadllm_kv_tile_varlen", vp.data_ptr(), hk * D, D, cu.data_ptr(), B, hk, Lmax, D,
                          vt.data_ptr(), nbytes, s)
                nblk = -(-Lmax // 64)
                out = torch.empty(R, hq * D, dtype=BF16, device=self.device)
                gate = P[:, D:]
                _lib.call("kadllm_attention_tiled_varlen", q.data_ptr(), hq * D, 0, D, kt.data_ptr(), vt.data_ptr(),
                          nblk, None, 0, 0, 0, None, 0, 0, 0, gate.data_ptr(), P.stride(0), 0, 2 * D,
                          out.data_ptr(), out.stride(0), 0, D, self.status.data_ptr(), cu.data_ptr(), B, 1, 1, 0, hq,
                          hk, Lmax, D, D ** -0.5, 1, s)
                w_post = m.w_o
                prefix.append((kp, vp))
                tiles.append((kt, vt, nblk))
            if i + 1 < len(self.layers):
                self._post_mixer(layer, out, w_post, x, normed, self.layers[i + 1].input_ln)
        last = self._finish_last_rows(layer, out, w_post, x, cu[1:].long() - 1)
        logits = self._gemm(last, self.lm_head if head is None else head)
        return logits, HybridPrefix(Lmax, B, self.owner, tuple(prefix), tuple(tiles), cu, tuple(lens))

    # ------------------------------------------------------------------ decode
    @torch.no_grad()
    def decode_hidden(self, history: torch.Tensor, state: HybridPrefix, cache: dict | None = None,
                      reuse: tuple | None = None) -> torch.Tensor:
        """Replay history [B, W, T] -> final-norm hidden of the last position [B*W, H].

        ``cache`` (a dict; T = 1) receives what a following two-token step of these
        beams' children reuses: per GDN layer the projection rows of the token, per
        attention layer its q / k / v.  ``reuse = (cache, parent, prev_width)`` (T = 2):
        the first suffix token of beam j of request b is the token of the previous
        step's beam ``parent[b, j]`` (int32), whose per-layer work the cache holds;
        only the new token is replayed (its projections, the continuing GDN mixer,
        attention with the first token's q / k / v gathered by parent, MLP)."""
        if reuse is not None:
            return self._decode_continue(history, state, *reuse)
        c = self.cfg
        B, W, T = history.shape
        BW, R = B * W, B * W * T
        ids = history.to(device=self.device, dtype=torch.int64).reshape(-1).contiguous()
        x, normed = self._embed(ids)
        s = self._stream()
        hk, D, hq = c.num_key_value_heads, c.head_dim, c.num_attention_heads
        varlen = state.cu is not None
        pos = None
        if varlen:  # suffix position of row (b, w, t): the request's own prefix length + t
            lens = torch.tensor(state.lengths, dtype=torch.int64)
            pos = (lens.repeat_interleave(W * T) + torch.arange(T, dtype=torch.int64).repeat(B * W)).to(self.device)
        for i, (layer, cached) in enumerate(zip(self.layers, state.layers)):
            m = layer.mixer
            P = self._gemm(normed, m.w_in)
            if layer.kind == LINEAR:
                out = torch.empty(R, c.value_dim, dtype=BF16, device=self.device)
                conv_state, rec = cached
                # the first decode step keeps each beam's k, delta and decay for the next step
                records = None
                if cache is not None and T == 1 and self._mixer_records_ok():
                    records = torch.empty(_lib.lib().kadllm_gdn_mixer_record_bytes(
                        B, W, c.linear_num_value_heads, c.linear_value_head_dim), dtype=torch.uint8, device=self.device)
                _lib.call("kadllm_gdn_mixer_replay", P.data_ptr(), P.stride(0), conv_state.data_ptr(),
                          conv_state.shape[-1], m.conv_w.data_ptr(), rec.data_ptr(), m.a_log.data_ptr(),
                          m.dt_bias.data_ptr(), m.norm_w.data_ptr(), c.rms_norm_eps, out.data_ptr(), B, W, T,
                          c.linear_num_key_heads, c.linear_num_value_heads, c.linear_key_head_dim,
                          c.linear_value_head_dim, _lib.ptr(records), self.status.data_ptr(), s)
                if cache is not None:
                    cache[i] = (P, records)
                self._gemm(out, m.w_out, resid=x)
            else:
                q = torch.empty(R, hq, D, dtype=BF16, device=self.device)
                ks = torch.empty(R, hk, D, dtype=BF16, device=self.device)
                vs = torch.empty_like(ks)
                suffix_strides = (T * hk * D, hk * D, D)  # (beam row, step, head)
                if varlen:
                    self._qk_rope(P, R, 0, T, q, ks, suffix_strides, vs, suffix_strides, m, pos_of_row=pos,
                                  max_pos=state.length + T)
                else:
                    self._qk_rope(P, R, state.length, T, q, ks, suffix_strides, vs, suffix_strides, m)
                if cache is not None:
                    cache[i] = (q.view(R, hq * D), ks.view(R, hk * D), vs.view(R, hk * D))
                out = torch.empty(R, hq * D, dtype=BF16, device=self.device)
                self._attend(i, state, q, ks, vs, P, out, B, W, T, T * P.stride(0), P.stride(0))
                self._gemm(out, m.w_o, resid=x)
            self._add_norm(x, None, layer.post_ln, normed)
            self._mlp(layer, normed, x)
            if i + 1 < len(self.layers):
                self._add_norm(x, None, self.layers[i + 1].input_ln, normed)
        last = torch.empty(BW, c.hidden_size, dtype=BF16, device=self.device)
        self._add_norm(x, None, self.final_norm, last, rows=BW, step=T, offset=T - 1)
        return last

    def _attend(self, i, state, q, ks, vs, P, out, B, W, T, sg_row, sg_t, t0=0):
        """Decode attention of layer i: rows (beam, t) of q [B*W, T, Hq, D] against the
        request's prefix and the beam's suffix keys ks / vs [B*W, T, HK, D] (row-major
        views), the output gate from P (gate row stride sg_row per beam, sg_t per step),
        into out [B*W, T, Hq*D]; only steps t >= t0 have queries and outputs."""
        c = self.cfg
        hk, D, hq = c.num_key_value_heads, c.head_dim, c.num_attention_heads
        s = self._stream()
        suffix_strides = (T * hk * D, hk * D, D)
        gate = P[:, D:]  # gate of head h at column h*2D + D
        tile = state.tiles[i] if i < len(state.tiles) else None
        pk, pv = state.layers[i]  # [B, L, HK, D] views
        if state.cu is not None:  # every request against its own prefix length
            kt, vt, nblk = tile
            _lib.call("kadllm_attention_tiled_varlen", q.data_ptr(), T * hq * D, hq * D, D, kt.data_ptr(),
                      vt.data_ptr(), nblk, ks.data_ptr(), *suffix_strides, vs.data_ptr(), *suffix_strides,
                      gate.data_ptr(), sg_row, sg_t, 2 * D, out.data_ptr(), T * hq * D, hq * D, D,
                      self.status.data_ptr(), state.cu.data_ptr(), B, W, T, t0, hq, hk, state.length, D, D ** -0.5, 0, s)
        elif tile is not None:
            kt, vt, nblk = tile
            _lib.call("kadllm_attention_tiled", q.data_ptr(), T * hq * D, hq * D, D, kt.data_ptr(),
                      vt.data_ptr(), nblk, ks.data_ptr(), *suffix_strides, vs.data_ptr(), *suffix_strides,
                      gate.data_ptr(), sg_row, sg_t, 2 * D, out.data_ptr(), T * hq * D, hq * D, D,
                      self.status.data_ptr(), B, W, T, t0, hq, hk, state.length, D, D ** -0.5, 0, s)
        else:
            if t0:
                raise NotImplementedError("query steps after the first need the tiled (head dim 256) attention")
            _lib.call("kadllm_prefix_attention", q.data_ptr(), T * hq * D, hq * D, D, pk.data_ptr(),
                      *pk.stride()[:3], pv.data_ptr(), *pv.stride()[:3], ks.data_ptr(), *suffix_strides,
                      vs.data_ptr(), *suffix_strides, None, gate.data_ptr(), sg_row, sg_t, 2 * D, out.data_ptr(),
                      T * hq * D, hq * D, D, _lib.DTYPE_CODES[BF16], B, W, T, hq, hk, state.length, D, D ** -0.5, s)

    def _decode_continue(self, history, state, prev, parent, prev_width):
        """The T = 2 step from the previous (T = 1) step's cache: rows are the new tokens only."""
        c = self.cfg
        B, W, T = history.shape
        if T != 2:
            raise ValueError("step reuse continues a one-token suffix by one token (T = 2)")
        R = B * W
        parent = parent.to(device=self.device, dtype=torch.int32).reshape(-1).contiguous()
        if parent.numel() != R:
            raise ValueError("parent must hold one previous-beam index per beam")
        ids = history[:, :, -1].to(device=self.device, dtype=torch.int64).reshape(-1).contiguous()
        x, normed = self._embed(ids)
        s = self._stream()
        hk, D, hq = c.num_key_value_heads, c.head_dim, c.num_attention_heads
        pos = None
        if state.cu is not None:
            pos = (torch.tensor(state.lengths, dtype=torch.int64) + 1).repeat_interleave(W).to(self.device)
        for i, (layer, cached) in enumerate(zip(self.layers, state.layers)):
            m = layer.mixer
            P = self._gemm(normed, m.w_in)
            if layer.kind == LINEAR:
                out = torch.empty(R, c.value_dim, dtype=BF16, device=self.device)
                conv_state, rec = cached
                P0, records = prev[i]  # the previous step's projection rows and records (or None)
                _lib.call("kadllm_gdn_mixer_continue", P0.data_ptr(), parent.data_ptr(), prev_width, P.data_ptr(),
                          P.stride(0), conv_state.data_ptr(), conv_state.shape[-1], m.conv_w.data_ptr(),
                          rec.data_ptr(), m.a_log.data_ptr(), m.dt_bias.data_ptr(), m.norm_w.data_ptr(),
                          c.rms_norm_eps, out.data_ptr(), B, W, c.linear_num_key_heads, c.linear_num_value_heads,
                          c.linear_key_head_dim, c.linear_value_head_dim, _lib.ptr(records), self.status.data_ptr(),
                          s)
                self._gemm(out, m.w_out, resid=x)
            else:
                q = torch.empty(R, 2, hq, D, dtype=BF16, device=self.device)
                ks = torch.empty(R, 2, hk, D, dtype=BF16, device=self.device)
                vs = torch.empty_like(ks)
                pq, pk, pv = prev[i]  # the first token's q / k / v, rows of the previous step's beams
                self._gather_rows(pq, parent, W, prev_width, q, 2 * hq * D)
                self._gather_rows(pk, parent, W, prev_width, ks, 2 * hk * D)
                self._gather_rows(pv, parent, W, prev_width, vs, 2 * hk * D)
                kv_strides = (2 * hk * D, hk * D, D)  # (beam row, step, head) of slot 1
                if pos is not None:
                    self._qk_rope(P, R, 0, 1, q[:, 1], ks[:, 1], kv_strides, vs[:, 1], kv_strides, m,
                                  pos_of_row=pos, max_pos=state.length + 2, q_row_stride=2 * hq * D)
                else:
                    self._qk_rope(P, R, state.length + 1, 1, q[:, 1], ks[:, 1], kv_strides, vs[:, 1], kv_strides,
                                  m, q_row_stride=2 * hq * D)
                out = torch.empty(R, 2, hq * D, dtype=BF16, device=self.device)
                if state.tiles and state.tiles[i] is not None:  # queries of the new token only
                    self._attend(i, state, q, ks, vs, P, out, B, W, 2, P.stride(0), 0, t0=1)
                else:  # the first token's query rows are recomputed alongside (outputs unused)
                    self._attend(i, state, q, ks, vs, P, out, B, W, 2, P.stride(0), 0)
                self._gemm(out[:, 1], m.w_o, resid=x)
            self._add_norm(x, None, layer.post_ln, normed)
            self._mlp(layer, normed, x)
            if i + 1 < len(self.layers):
                self._add_norm(x, None, self.layers[i + 1].input_ln, normed)
        last = torch.empty(R, c.hidden_size, dtype=BF16, device=self.device)
        self._add_norm(x, None, self.final_norm, last, rows=R)
        return last

    @torch.no_grad()
    def decode(self, history: torch.Tensor, state: HybridPrefix, head: torch.Tensor | None = None,
               cache: dict | None = None, reuse: tuple | None = None,
               select_workspace: torch.Tensor | None = None) -> torch.Tensor:
        """Replay [B, W, T] suffix tokens; return [B, W, V] logits (BF16) over the LM
        head's rows, or over ``head``'s rows when given (``cache`` / ``reuse``: see
        :meth:`decode_hidden`).  With ``select_workspace`` (a selector's workspace) the
        LM head also writes each row's chunk statistics there for the fused selection."""
        B, W, _ = history.shape
        w = self.lm_head if head is None else head
        hidden = self.decode_hidden(history, state, cache=cache, reuse=reuse)
        if select_workspace is None:
            return self._gemm(hidden, w).view(B, W, -1)
        V = w.shape[0]
        logits = torch.empty(B * W, V, dtype=BF16, device=self.device)
        _lib.call("kadllm_gemm_logits", hidden.data_ptr(), hidden.stride(0), w.data_ptr(), w.stride(0),
                  logits.data_ptr(), V, B * W, V, hidden.shape[1], select_workspace.data_ptr(),
                  select_workspace.numel(), B, W, self.status.data_ptr(), self._stream())
        return logits.view(B, W, V)
