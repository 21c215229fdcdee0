"""Independent numpy restatement of the reference decode step, used to check the
C oracle's model logic on tiny shapes (fp64 accumulation, bf16 rounding at the
points where the reference materialises a bf16 Tensor; llama_model.cpp:103-238,
qwen_model.cpp:73-146, qwen_adapter_model.cpp:22-43)."""
import numpy as np

from oracle import bf16_to_f32, f32_to_bf16


def rb(x):
    """round to bf16 and back (fp32 values)"""
    return bf16_to_f32(f32_to_bf16(np.asarray(x, np.float32)))


def rope_freqs(hd, theta):
    i = np.arange(hd // 2, dtype=np.float32)
    return (np.float32(1.0) / np.power(np.float32(theta), (np.float32(2.0) * i) / np.float32(hd))).astype(np.float32)


class NumpyModel:
    def __init__(self, kw, weights, lora=None):
        self.kw = kw
        self.w = {k: bf16_to_f32(v).astype(np.float64) for k, v in weights.items()}
        self.lora = lora  # dict(rank, alpha, w={name: uint16})
        self.k = [[] for _ in range(kw["n_layers"])]
        self.v = [[] for _ in range(kw["n_layers"])]
        self.freqs = rope_freqs(kw.get("head_dim", kw["hidden"] // kw["n_heads"]), kw["rope_theta"])

    def _lin(self, x, name):
        return rb(x.astype(np.float64) @ self.w[name].T)

    def _norm(self, x, name):
        eps = self.kw["rms_eps"]
        ss = (x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True)
        scale = 1.0 / np.sqrt(ss.astype(np.float32) + np.float32(eps))
        return rb(x * scale.astype(np.float32) * self.w[name].astype(np.float32))

    def _lora(self, x, li, proj, y):
        if not self.lora:
            return y
        base = f"layers.{li}.{proj}"
        if base + ".lora_A" not in self.lora["w"]:
            return y
        A = bf16_to_f32(self.lora["w"][base + ".lora_A"]).astype(np.float64)
        B = bf16_to_f32(self.lora["w"][base + ".lora_B"]).astype(np.float64)
        down = rb(x.astype(np.float64) @ A.T)
        up = rb(down.astype(np.float64) @ B.T)
        delta = rb(up * np.float32(self.lora["alpha"] / self.lora["rank"]))
        return rb(y + delta)

    def _rope(self, x, pos):
        hd = x.shape[-1]
        half = hd // 2
        ang = (np.float32(pos) * self.freqs).astype(np.float32)
        c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
        x0, x1 = x[..., :half], x[..., half:]
        return rb(np.concatenate([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1))

    def step(self, tok):
        kw = self.kw
        H, nq, nkv = kw["hidden"], kw["n_heads"], kw.get("n_kv_heads", kw["n_heads"])
        hd = kw.get("head_dim", H // nq)
        pos = len(self.k[0])
        h = bf16_to_f32(f32_to_bf16(self.w["model.embed_tokens.weight"][tok].astype(np.float32)))
        for li in range(kw["n_layers"]):
            p = f"model.layers.{li}."
            n1 = self._norm(h, p + "input_layernorm.weight")
            qkv = []
            for j, nm in enumerate(("q_proj", "k_proj", "v_proj")):
                y = self._lin(n1, p + f"self_attn.{nm}.weight")
                if kw.get("qkv_bias"):
                    y = rb(y + self.w[p + f"self_attn.{nm}.bias"].astype(np.float32))
                qkv.append(self._lora(n1, li, f"self_attn.{nm}", y))
            q = self._rope(qkv[0].reshape(nq, hd), pos)
            k = self._rope(qkv[1].reshape(nkv, hd), pos)
            v = qkv[2].reshape(nkv, hd)
            self.k[li].append(k)
            self.v[li].append(v)
            K = np.stack(self.k[li]).astype(np.float64)  # [T, nkv, hd]
            Vv = np.stack(self.v[li]).astype(np.float64)
            out = np.empty((nq, hd), np.float32)
            g = nq // nkv
            for hh in range(nq):
                kh = hh // g
                sc = (K[:, kh, :] @ q[hh].astype(np.float64)) * (1.0 / np.sqrt(hd))
                sc = sc - sc.max()
                pr = np.exp(sc)
                pr /= pr.sum()
                out[hh] = (pr @ Vv[:, kh, :]).astype(np.float32)
            attn = rb(out.reshape(-1))
            o = self._lora(attn, li, "self_attn.o_proj", self._lin(attn, p + "self_attn.o_proj.weight"))
            r1 = rb(h + o)
            n2 = self._norm(r1, p + "post_attention_layernorm.weight")
            gt = self._lora(n2, li, "mlp.gate_proj", self._lin(n2, p + "mlp.gate_proj.weight"))
            up = self._lora(n2, li, "mlp.up_proj", self._lin(n2, p + "mlp.up_proj.weight"))
            act = rb(rb(gt / (1.0 + np.exp(-gt.astype(np.float64)))) * up)
            dn = self._lora(act, li, "mlp.down_proj", self._lin(act, p + "mlp.down_proj.weight"))
            h = rb(r1 + dn)
        hn = self._norm(h, "model.norm.weight")
        return (hn.astype(np.float64) @ self.w["lm_head.weight"].T).astype(np.float32)
