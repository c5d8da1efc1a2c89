"""Generate the golden fixtures under tests/golden/ by running the REFERENCE.

Run in a container where the Kadllm reference sources and Transformers are
importable (pass the reference's ``src`` directory as the first argument):

    python tests/golden/make_golden.py <kadllm-src-dir>              # the small fixtures
    python tests/golden/make_golden.py <kadllm-src-dir> --headline   # the 0.8B-sized fixtures

Every fixture records inputs and the reference's outputs:

* ``model_<dtype>.npz``  tiny hybrid (the CPU-plumbing config) through
  ``Qwen35GRBeamAdapter`` (torch backends) + ``grbeam_search`` with widths
  [8, 8, 8]: prefill logits, every prefix tensor, decode logits for both decode
  steps (all beams) and for fixed histories of 1-3 tokens shared by both dtypes,
  final tokens / scores / valid.  Weights are regenerated
  from ``kadllm_b200.synthetic.numpy_weights(TINY, seed=0, init="test")``.
* ``ops_<dtype>.npz``    seeded inputs and outputs of ``kadllm.ops.gated_delta``,
  ``causal_conv1d`` and ``prefix_attention`` (torch paths), including a masked
  prefix with a fully masked request, and of Transformers'
  ``torch_chunk_gated_delta_rule`` (prefill scan, with final state).
* ``select.npz``         ``grbeam_search`` driven by a fixed-logits adapter
  (ties, a mask via ``allowed``, and an all-masked beam).
* ``headline_<dtype>.npz`` the benchmark's 0.8B-shaped model, batch 2, prompt
  1024, widths [256, 256, 256] (see ``headline``).

The reference is not available where the GPU tests run; these files are.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))


def main(ref_src: str) -> None:
    sys.path.insert(0, ref_src)
    from kadllm import grbeam_search
    from kadllm.adapters import Qwen35GRBeamAdapter
    from kadllm.ops import causal_conv1d, gated_delta, prefix_attention
    from transformers import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import (
        Qwen3_5TextModel,
        torch_chunk_gated_delta_rule,
    )

    from kadllm_b200.config import TINY
    from kadllm_b200.synthetic import numpy_weights, random_prompts

    torch.set_num_threads(1)
    torch.set_grad_enabled(False)
    dtypes = {"fp32": torch.float32, "bf16": torch.bfloat16}

    # ------------------------------------------------------------ model
    for name, tdt in dtypes.items():
        cfg = TINY
        w = numpy_weights(cfg, seed=0, init="test")
        model = Qwen3_5TextModel._from_config(Qwen3_5TextConfig(**cfg.to_hf_kwargs()), dtype=tdt).eval()
        model.load_state_dict({k: torch.from_numpy(v).to(tdt) for k, v in w.items()}, strict=True)
        head = torch.nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False).eval()
        head.weight = model.embed_tokens.weight
        adapter = Qwen35GRBeamAdapter(model, head)
        ids = random_prompts(2, 64, cfg.vocab_size, seed=0)
        tids = torch.from_numpy(ids)
        widths = [8, 8, 8]
        res = grbeam_search(adapter, tids, widths)
        pre = adapter.prefill(tids)
        out = dict(ids=ids, widths=np.array(widths), tokens=res.tokens.numpy(),
                   scores=res.scores.float().numpy(), valid=res.valid.numpy(),
                   prefill_logits=pre.logits.float().numpy())
        for i, (a, b) in enumerate(pre.state.layers):
            out[f"layer{i}_a"] = a.float().numpy()
            out[f"layer{i}_b"] = b.float().numpy()
        hist1 = res.tokens[:, :, :1]
        hist2 = res.tokens[:, :, :2]
        out["decode1_history"] = hist1.numpy()
        out["decode1_logits"] = adapter.decode(hist1, pre.state).float().numpy()
        out["decode2_history"] = hist2.numpy()
        out["decode2_logits"] = adapter.decode(hist2, pre.state).float().numpy()
        # the same fixed histories in both dtypes, so BF16 error can be measured against fp32
        fixed = np.random.default_rng(7).integers(0, cfg.vocab_size, (2, 8, 3))
        for T in (1, 2, 3):
            out[f"fixed{T}_history"] = fixed[:, :, :T]
            out[f"fixed{T}_logits"] = adapter.decode(torch.from_numpy(fixed[:, :, :T]), pre.state).float().numpy()
        np.savez_compressed(HERE / f"model_{name}.npz", **out)
        print("model", name, res.scores[0].tolist())

    # ------------------------------------------------------------ ops
    for name, tdt in dtypes.items():
        rng = np.random.default_rng(1)
        f = lambda *s, scale=1.0: (scale * rng.standard_normal(s)).astype(np.float32)
        t = lambda a: torch.from_numpy(a).to(tdt)
        out = {}
        # gated delta replay: B=2, W=3, T=3, H=2, HV=4, K=V=32
        B, W, T, H, HV, K = 2, 3, 3, 2, 4, 32
        q, k, v = f(B * W, T, H, K), f(B * W, T, H, K), f(B * W, T, HV, K)
        g = -rng.uniform(0.0, 1.0, (B * W, T, HV)).astype(np.float32)
        beta = rng.uniform(0.0, 1.0, (B * W, T, HV)).astype(np.float32)
        s0 = f(B, HV, K, K, scale=0.5)
        qt, kt, vt, st = t(q), t(k), t(v), t(s0)
        o = gated_delta(qt, kt, vt, torch.from_numpy(g), torch.from_numpy(beta), st,
                        beam_width=W, backend="torch")
        out.update(gd_q=qt.float().numpy(), gd_k=kt.float().numpy(), gd_v=vt.float().numpy(),
                   gd_g=g, gd_beta=beta, gd_s0=st.float().numpy(), gd_out=o.float().numpy(),
                   gd_W=np.array(W))
        # causal conv replay: B=2, W=3, C=48, T=3, hist=4
        C = 48
        x, cs, cw = f(B * W, C, T), f(B, C, 4), f(C, 4, scale=0.5)
        o = causal_conv1d(t(x), t(cs), t(cw), beam_width=W, backend="torch")
        out.update(cv_x=t(x).float().numpy(), cv_state=t(cs).float().numpy(),
                   cv_w=t(cw).float().numpy(), cv_out=o.float().numpy(), cv_W=np.array(W))
        # prefix attention: B=2, W=3, T=3, H=4, HK=2, D=32, L=9, plus a masked variant
        H, HK, D, L = 4, 2, 32, 9
        aq, pk, pv = f(B * W, T, H, D), f(B, L, HK, D), f(B, L, HK, D)
        sk, sv = f(B * W, T, HK, D), f(B * W, T, HK, D)
        o = prefix_attention(t(aq), t(pk), t(pv), t(sk), t(sv), beam_width=W, backend="torch")
        mask = np.ones((B, L), bool)
        mask[0, 5:] = False
        mask[1, :] = False
        om = prefix_attention(t(aq), t(pk), t(pv), t(sk), t(sv), beam_width=W, backend="torch",
                              prefix_mask=torch.from_numpy(mask))
        e = prefix_attention(t(aq), t(pk)[:, :0], t(pv)[:, :0], t(sk), t(sv), beam_width=W,
                             backend="torch")
        out.update(at_q=t(aq).float().numpy(), at_pk=t(pk).float().numpy(),
                   at_pv=t(pv).float().numpy(), at_sk=t(sk).float().numpy(),
                   at_sv=t(sv).float().numpy(), at_out=o.float().numpy(), at_mask=mask,
                   at_out_masked=om.float().numpy(), at_out_empty=e.float().numpy(),
                   at_W=np.array(W))
        # chunked prefill scan: B=2, L=100 (ragged last chunk), HV=2, K=V=32
        Lp, Hs = 100, 2
        cq, ck, cvv = f(2, Lp, Hs, K), f(2, Lp, Hs, K), f(2, Lp, Hs, K)
        cg = -rng.uniform(0.0, 0.5, (2, Lp, Hs)).astype(np.float32)
        cb = rng.uniform(0.0, 1.0, (2, Lp, Hs)).astype(np.float32)
        co, cstate = torch_chunk_gated_delta_rule(
            t(cq), t(ck), t(cvv), g=torch.from_numpy(cg), beta=t(cb), initial_state=None,
            output_final_state=True, use_qk_l2norm_in_kernel=True)
        out.update(ch_q=t(cq).float().numpy(), ch_k=t(ck).float().numpy(),
                   ch_v=t(cvv).float().numpy(), ch_g=cg, ch_beta=t(cb).float().numpy(),
                   ch_out=co.float().numpy(), ch_state=cstate.float().numpy())
        np.savez_compressed(HERE / f"ops_{name}.npz", **out)
        print("ops", name)

    # ------------------------------------------------------------ selection
    from kadllm.grbeam import PrefillResult

    rng = np.random.default_rng(2)
    B, V = 3, 64
    coarse = (np.round(rng.standard_normal((8, B, 4, V)) * 4) / 4).astype(np.float32)  # many exact ties
    smooth = (3 * rng.standard_normal((8, B, 4, V))).astype(np.float32)  # no ties

    def fixed_adapter(steps):
        class FixedAdapter:
            def prefill(self, ids):
                return PrefillResult(torch.from_numpy(steps[0, :, 0].copy()), None)

            def decode(self, history, state):
                Wc = history.shape[1]
                return torch.from_numpy(steps[history.shape[2], :, :Wc].copy())

        return FixedAdapter()

    def allowed(history, logits):
        m = torch.ones_like(logits, dtype=torch.bool)
        m[..., 1::3] = False
        if history.shape[2] >= 1:
            m[:, 0, :] = False  # first beam fully masked
        return m

    ids = torch.zeros(B, 5, dtype=torch.long)
    out = dict(coarse=coarse, smooth=smooth)
    for name, steps in (("coarse", coarse), ("smooth", smooth)):
        r1 = grbeam_search(fixed_adapter(steps), ids, [4, 4, 3])
        r2 = grbeam_search(fixed_adapter(steps), ids, [4, 4, 4], allowed=allowed)
        out.update({f"{name}_tokens": r1.tokens.numpy(), f"{name}_scores": r1.scores.numpy(),
                    f"{name}_valid": r1.valid.numpy(), f"{name}_masked_tokens": r2.tokens.numpy(),
                    f"{name}_masked_scores": r2.scores.numpy(),
                    f"{name}_masked_valid": r2.valid.numpy()})
    np.savez_compressed(HERE / "select.npz", **out)
    print("select", out["smooth_scores"].tolist())


HEADLINE_WIDTHS = [256, 256, 256]
HEADLINE_BATCH, HEADLINE_PROMPT = 2, 1024


def headline(ref_src: str) -> None:
    """The benchmark's model at its real size (Qwen3.5-0.8B-shaped: 24 layers,
    hidden 1024, vocabulary 248,320) through the reference's torch path, in BF16
    and fp32 with the same (BF16-valued) weights: ``headline_<dtype>.npz``.

    Weights: ``kadllm_b200.synthetic.torch_weights(QWEN35_08B, seed=0,
    device="cpu")`` (the benchmark's distributions, drawn by torch's CPU
    generator, so the GPU test regenerates them bit-identically).  Prompts:
    ``random_prompts(2, 1024, vocab, seed=0)``.  Recorded: the final beams
    (tokens, scores, valid) of ``grbeam_search`` with widths [256, 256, 256]; the
    hidden state of the last prompt position after every decoder layer (forward
    hooks on the prefill) and after the final norm; the first-token logits; for
    the fixed histories ``tokens[:, :, :2]`` of the BF16 search (in both files,
    so the BF16 results can be measured against fp32 at the same histories),
    the final-norm hidden of the last position of beams 0-7 and the logits of
    beams 0-1 of every request.  Logits are stored as BF16 bit patterns
    (``*_bits``, uint16) in the BF16 file and as fp32 in the fp32 file (request 0
    / beam 0 only) to keep the files small.
    """
    sys.path.insert(0, ref_src)
    from kadllm import grbeam_search
    from kadllm.adapters import Qwen35GRBeamAdapter
    from transformers import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextModel

    from kadllm_b200.config import QWEN35_08B
    from kadllm_b200.synthetic import random_prompts, torch_weights

    torch.set_num_threads(__import__("os").cpu_count() or 1)
    torch.set_grad_enabled(False)
    cfg = QWEN35_08B
    w = torch_weights(cfg, seed=0, device="cpu")  # BF16 values
    ids = random_prompts(HEADLINE_BATCH, HEADLINE_PROMPT, cfg.vocab_size, seed=0)
    tids = torch.from_numpy(ids)
    for name, tdt in (("bf16", torch.bfloat16), ("fp32", torch.float32)):
        model = Qwen3_5TextModel._from_config(Qwen3_5TextConfig(**cfg.to_hf_kwargs()), dtype=tdt).eval()
        model.load_state_dict({k: v.to(tdt) for k, v in w.items()}, strict=True)
        head = torch.nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False).eval()
        head.weight = model.embed_tokens.weight
        adapter = Qwen35GRBeamAdapter(model, head)
        taps = []
        hooks = [layer.register_forward_hook(lambda m, a, out: taps.append(out[:, -1].float().clone()))
                 for layer in model.layers]
        pre = adapter.prefill(tids)
        for h in hooks:
            h.remove()
        final = model.norm(taps[-1].to(tdt)).float()
        res = grbeam_search(adapter, tids, HEADLINE_WIDTHS)
        if tdt == torch.bfloat16:  # both files decode at the BF16 search's histories
            hist2 = res.tokens[:, :, :2].contiguous()
        normed = []
        hook = model.norm.register_forward_hook(lambda m, a, out: normed.append(out.float().clone()))
        dec = adapter.decode(hist2, pre.state)
        hook.remove()
        dec_hidden = normed[0].reshape(HEADLINE_BATCH, -1, cfg.hidden_size)[:, :8]
        out = dict(ids=ids, widths=np.array(HEADLINE_WIDTHS), tokens=res.tokens.numpy(),
                   scores=res.scores.float().numpy(), valid=res.valid.numpy(),
                   layer_hidden=torch.stack(taps).numpy(), final_hidden=final.numpy(),
                   decode_history=hist2.numpy(), decode_hidden=dec_hidden.numpy())
        if tdt == torch.bfloat16:
            out["prefill_logits_bits"] = pre.logits.view(torch.int16).numpy().view(np.uint16)
            out["decode_logits_bits"] = dec[:, :2].contiguous().view(torch.int16).numpy().view(np.uint16)
        else:
            out["prefill_logits0"] = pre.logits[0].numpy()
            out["decode_logits00"] = dec[0, 0].numpy()
        np.savez_compressed(HERE / f"headline_{name}.npz", **out)
        print("headline", name, res.scores[:, :4].tolist(), res.scores[:, -1].tolist(), flush=True)
        del model, adapter, pre, res, dec


if __name__ == "__main__":
    if len(sys.argv) == 3 and sys.argv[2] == "--headline":
        headline(sys.argv[1])
    elif len(sys.argv) == 2:
        main(sys.argv[1])
    else:
        raise SystemExit(__doc__)
