"""A random-init Qwen2 + NF4 + LoRA model with the attribute layout of a PEFT-wrapped,
bitsandbytes-4-bit HF Qwen2ForCausalLM — the objects the fused step reads (the reference reads
them duck-typed too: solution/engine.py:77-101, 875-915, 1571-1597).

bitsandbytes and peft are not installed here, so this module stands in for them: each projection
is a `LoraLinear` (lora_A / lora_B / scaling / lora_dropout / active_adapters) around a
`Linear4bit` whose `weight` carries `.data` (the packed NF4 bytes, element i in byte i // 2, high
nibble first) and `.quant_state` (code, blocksize 64, absmax, nested state2 / offset, shape,
quant_type "nf4"). The quantiser picks the nearest NF4 level of w / absmax per 64-block: valid
NF4 bytes, not bitsandbytes' own quantiser (which is not on the training hot path).
"""

import math
from dataclasses import dataclass

import torch

NF4_LEVELS = (-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
              -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
              0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
              0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0)


@dataclass
class Qwen2Config:
    vocab_size: int = 151936
    hidden_size: int = 1536
    intermediate_size: int = 8960
    num_hidden_layers: int = 28
    num_attention_heads: int = 12
    num_key_value_heads: int = 2
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    tie_word_embeddings: bool = True
    model_type: str = "qwen2"
    hidden_act: str = "silu"
    use_sliding_window: bool = False


QWEN25_1P5B = Qwen2Config()
QWEN25_7B = Qwen2Config(vocab_size=152064, hidden_size=3584, intermediate_size=18944,
                        num_attention_heads=28, num_key_value_heads=4,
                        tie_word_embeddings=False)
TINY = Qwen2Config(vocab_size=3000, hidden_size=256, intermediate_size=640, num_hidden_layers=2,
                   num_attention_heads=4, num_key_value_heads=2, head_dim=64)


# ---------------------------------------------------------------------------------------------
# NF4 quantisation (setup only)
# ---------------------------------------------------------------------------------------------
class State2:
    def __init__(self, code, absmax, blocksize):
        self.code, self.absmax, self.blocksize = code, absmax, blocksize


class QuantState:
    """The fields of a bitsandbytes QuantState the fused step reads."""

    def __init__(self, absmax, shape, code, blocksize=64, nested=False, state2=None, offset=None,
                 dtype=torch.float16):
        self.absmax, self.shape, self.code, self.blocksize = absmax, torch.Size(shape), code, blocksize
        self.nested, self.state2, self.offset, self.dtype = nested, state2, offset, dtype
        self.quant_type = "nf4"


class Params4bit:
    """Stands in for bnb.nn.Params4bit: .data = packed bytes [numel / 2, 1] uint8."""

    def __init__(self, data, quant_state):
        self.data, self.quant_state = data, quant_state
        self.requires_grad = False

    @property
    def device(self):
        return self.data.device


def nested_code(device):
    """A signed 256-level table for double-quantised absmax (not bitsandbytes' dynamic map)."""
    pos = torch.logspace(-4, 0, 127, dtype=torch.float64)
    code = torch.cat([-pos.flip(0), torch.zeros(1, dtype=torch.float64), pos,
                      torch.ones(1, dtype=torch.float64)])
    return code.sort().values.float().to(device)


def quantize_nf4(w, nested=False, bs2=256):
    """w [rows, cols] (any float dtype, on its device) -> Params4bit with NF4 bytes."""
    rows, cols = w.shape
    dev = w.device
    blocks = w.float().reshape(-1, 64)
    absmax = blocks.abs().amax(dim=1)
    norm = blocks / torch.where(absmax > 0, absmax, torch.ones_like(absmax))[:, None]
    levels = torch.tensor(NF4_LEVELS, device=dev)
    mids = (levels[1:] + levels[:-1]) / 2
    q = torch.bucketize(norm.reshape(-1), mids).to(torch.uint8)
    packed = ((q[0::2] << 4) | q[1::2]).contiguous().view(-1, 1)
    code = levels.clone()
    if not nested:
        return Params4bit(packed, QuantState(absmax.contiguous(), (rows, cols), code))
    offset = absmax.mean()
    centred = absmax - offset
    nb2 = -(-centred.numel() // bs2)
    padded = torch.zeros(nb2 * bs2, device=dev)
    padded[:centred.numel()] = centred
    absmax2 = padded.view(nb2, bs2).abs().amax(dim=1)
    absmax2 = torch.where(absmax2 > 0, absmax2, torch.ones_like(absmax2))
    code2 = nested_code(dev)
    normed = centred / absmax2.repeat_interleave(bs2)[:centred.numel()]
    mids2 = (code2[1:] + code2[:-1]) / 2
    q2 = torch.bucketize(normed, mids2).to(torch.uint8)
    state = QuantState(q2.contiguous(), (rows, cols), code, nested=True,
                       state2=State2(code2, absmax2.contiguous(), bs2),
                       offset=offset.reshape(()).clone())
    return Params4bit(packed, state)


# ---------------------------------------------------------------------------------------------
# modules
# ---------------------------------------------------------------------------------------------
class Linear4bit(torch.nn.Module):
    def __init__(self, weight, bias=None):
        super().__init__()
        self.weight = weight  # Params4bit (not an nn.Parameter: frozen bytes)
        self.bias = bias
        self.out_features, self.in_features = weight.quant_state.shape


class LoraLinear(torch.nn.Module):
    """The attributes of a peft LoRA Linear the fused step reads."""

    def __init__(self, base, r, alpha, dropout, name="default"):
        super().__init__()
        self.base_layer = base
        self.lora_A = torch.nn.ModuleDict({name: torch.nn.Linear(base.in_features, r, bias=False)})
        self.lora_B = torch.nn.ModuleDict({name: torch.nn.Linear(r, base.out_features, bias=False)})
        self.scaling = {name: alpha / r}
        self.lora_dropout = torch.nn.ModuleDict({name: torch.nn.Dropout(dropout)})
        self.active_adapters = [name]
        self.merged = False
        self.disable_adapters = False


class RMSNorm(torch.nn.Module):
    def __init__(self, H, eps, device):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(H, device=device), requires_grad=False)
        self.variance_epsilon = eps


class RotaryEmbedding(torch.nn.Module):
    """HF Qwen2RotaryEmbedding's default rule: inv_freq = theta^(-2i/D), emb = cat(f, f)."""

    def __init__(self, D, theta, device):
        super().__init__()
        self.inv_freq = 1.0 / (theta ** (torch.arange(0, D, 2, device=device, dtype=torch.int64)
                                         .float() / D))

    def forward(self, x, position_ids):
        freqs = position_ids[..., None].float() * self.inv_freq.to(x.device)
        emb = torch.cat([freqs, freqs], dim=-1)
        return emb.cos().to(x.dtype), emb.sin().to(x.dtype)


class _NS(torch.nn.Module):
    pass


class CausalLM(torch.nn.Module):
    def __init__(self, config):
        super().__init__()
        self.config = config


class PeftModel(torch.nn.Module):
    def __init__(self, causal):
        super().__init__()
        self.base_model_ref = causal

    def get_base_model(self):
        return self.base_model_ref


def build_qwen2_qlora(config=QWEN25_1P5B, r=16, alpha=32, dropout=0.05, device="cuda",
                      seed=0, nested=False, embed_dtype=torch.float16, lora_b_std=0.02,
                      norm_noise=0.0, bias_std=0.02, layers_override=None):
    """A PeftModel-shaped random-init QLoRA Qwen2 on `device`: base weights N(0, 0.02) quantised
    to NF4, fp32 LoRA A (Kaiming-uniform) and B (N(0, lora_b_std)) on q_proj and v_proj.
    layers_override builds only that many decoder layers (a bounded CPU sample)."""
    g = torch.Generator(device=device).manual_seed(seed)
    H, I, D = config.hidden_size, config.intermediate_size, config.head_dim
    HQ, HKV = config.num_attention_heads, config.num_key_value_heads

    def randn(*shape, std=0.02):
        return torch.randn(*shape, device=device, generator=g) * std

    causal = CausalLM(config)
    inner = _NS()
    emb = torch.nn.Embedding(config.vocab_size, H, device=device, dtype=embed_dtype)
    emb.weight.requires_grad_(False)
    emb.weight.data.copy_(randn(config.vocab_size, H).to(embed_dtype))
    inner.embed_tokens = emb
    layers = torch.nn.ModuleList()
    n_layers = config.num_hidden_layers if layers_override is None else layers_override
    for _ in range(n_layers):
        layer = _NS()
        attn = _NS()
        mlp = _NS()
        shapes = {"q_proj": (HQ * D, H), "k_proj": (HKV * D, H), "v_proj": (HKV * D, H),
                  "o_proj": (H, HQ * D), "gate_proj": (I, H), "up_proj": (I, H),
                  "down_proj": (H, I)}
        for name, shape in shapes.items():
            bias = None
            if name in ("q_proj", "k_proj", "v_proj"):
                bias = torch.nn.Parameter(randn(shape[0], std=bias_std).to(embed_dtype),
                                          requires_grad=False)
            base = Linear4bit(quantize_nf4(randn(*shape), nested=nested), bias)
            mod = base
            if name in ("q_proj", "v_proj"):
                mod = LoraLinear(base, r, alpha, dropout).to(device)
                a = mod.lora_A["default"].weight
                bound = 1.0 / math.sqrt(H)
                with torch.no_grad():
                    a.copy_((torch.rand(a.shape, device=device, generator=g) * 2 - 1) * bound)
                    mod.lora_B["default"].weight.copy_(randn(*mod.lora_B["default"].weight.shape,
                                                             std=lora_b_std))
            (attn if name.endswith(("q_proj", "k_proj", "v_proj", "o_proj")) else mlp) \
                .add_module(name, mod)
        attn.scaling = D ** -0.5
        layer.self_attn = attn
        layer.mlp = mlp
        layer.input_layernorm = RMSNorm(H, config.rms_norm_eps, device)
        layer.post_attention_layernorm = RMSNorm(H, config.rms_norm_eps, device)
        if norm_noise:
            for nrm in (layer.input_layernorm, layer.post_attention_layernorm):
                nrm.weight.data.add_(randn(H, std=norm_noise))
        layers.append(layer)
    inner.layers = layers
    inner.norm = RMSNorm(H, config.rms_norm_eps, device)
    if norm_noise:
        inner.norm.weight.data.add_(randn(H, std=norm_noise))
    inner.rotary_emb = RotaryEmbedding(D, config.rope_theta, device)
    causal.model = inner
    head = _NS()
    if config.tie_word_embeddings:
        head.weight = emb.weight
    else:
        head.weight = torch.nn.Parameter(randn(config.vocab_size, H).to(embed_dtype),
                                         requires_grad=False)
    causal.lm_head = head
    model = PeftModel(causal)
    model.add_module("base", causal)
    return model


def move_to(model, device):
    """Moves a stand-in model built by build_qwen2_qlora (on the CPU, say, where every machine
    draws the same random numbers) to `device`: the NF4 bytes and quantisation state, biases,
    norms, embeddings, rotary frequencies and the LoRA weights (kept as the same Parameters, so
    their identity and requires_grad survive)."""
    causal = model.get_base_model()
    inner = causal.model
    with torch.no_grad():
        for p in model.parameters():
            p.data = p.data.to(device)
        for layer in inner.layers:
            for mod in (layer.self_attn.q_proj, layer.self_attn.k_proj, layer.self_attn.v_proj,
                        layer.self_attn.o_proj, layer.mlp.gate_proj, layer.mlp.up_proj,
                        layer.mlp.down_proj):
                base = getattr(mod, "base_layer", mod)
                w, qs = base.weight, base.weight.quant_state
                w.data = w.data.to(device)
                qs.absmax, qs.code = qs.absmax.to(device), qs.code.to(device)
                if qs.nested:
                    qs.state2.code = qs.state2.code.to(device)
                    qs.state2.absmax = qs.state2.absmax.to(device)
                    qs.offset = qs.offset.to(device)
        inner.rotary_emb.inv_freq = inner.rotary_emb.inv_freq.to(device)
    return model


def lora_parameters(model):
    """The trainable LoRA weights in the order the fused step returns their gradients."""
    return [p for p in model.parameters() if p.requires_grad]
