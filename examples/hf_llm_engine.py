"""Serve a Hugging Face causal LM through this package's paged engine.

    python examples/hf_llm_engine.py --model /models/Meta-Llama-3-8B-Instruct --prompt "Hello"
    python examples/hf_llm_engine.py --tiny          # a small random Llama, no checkpoint needed (CPU)

``create_ar_engine`` accepts the transformers model itself (as the reference's generic AR engine
factory does) and moves its weights into the shared decoder, so generation runs on the paged KV
cache and the sm_100a kernels when the device is a GPU.  To serve the checkpoint over HTTP
instead: ``sgl-omni serve --model-path <dir>``.
"""
import argparse
import asyncio

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", help="checkpoint directory of a Llama / Mistral / Qwen2 / Qwen3 / Qwen3-MoE model")
    ap.add_argument("--tiny", action="store_true", help="a small random Llama instead of a checkpoint")
    ap.add_argument("--prompt", default="Hello")
    ap.add_argument("--max-new-tokens", type=int, default=16)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args()

    import transformers

    from sglang_omni_b200.engines.ar import ARRequest
    from sglang_omni_b200.engines.omni.factory import create_ar_engine
    from sglang_omni_b200.sampling_params import SamplingParams

    if a.tiny:
        cfg = transformers.LlamaConfig(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                                       num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512)
        cfg.architectures = ["LlamaForCausalLM"]
        torch.manual_seed(0)
        hf = transformers.AutoModelForCausalLM.from_config(cfg).float().eval()
        ids = [1] + [ord(c) % 512 for c in a.prompt]
        decode = lambda toks: " ".join(map(str, toks))  # noqa: E731
    else:
        tok = transformers.AutoTokenizer.from_pretrained(a.model)
        hf = transformers.AutoModelForCausalLM.from_pretrained(a.model, torch_dtype=torch.bfloat16)
        ids = tok.apply_chat_template([{"role": "user", "content": a.prompt}], add_generation_prompt=True)
        decode = lambda toks: tok.decode(toks, skip_special_tokens=True)  # noqa: E731

    engine = create_ar_engine(hf, max_seq_len=1024, device=a.device, max_batch=8, use_graphs=a.device != "cpu")
    del hf

    async def run():
        try:
            req = ARRequest("r0", list(ids), SamplingParams(temperature=0.0), max_new_tokens=a.max_new_tokens)
            return await engine.generate("r0", req)
        finally:
            engine.stop()

    out = asyncio.run(run())
    print(decode(out.output_ids))


if __name__ == "__main__":
    main()
