"""Client of a running server (`sgl-omni serve ...`): a chat completion with streamed text and
speech chunks over SSE (the chunks are WAV files, concatenated here into one PCM track), then a
non-streaming `/v1/audio/speech` request.

    python examples/openai_client.py --url http://localhost:8000 --audio question.wav
"""
import argparse
import base64
import io
import json
import wave

import httpx


def _pcm_of(wav_bytes: bytes) -> tuple[bytes, int]:
    with wave.open(io.BytesIO(wav_bytes)) as w:
        return w.readframes(w.getnframes()), w.getframerate()


def main(args):
    body = {"messages": [{"role": "user", "content": args.prompt}], "stream": True, "max_tokens": args.max_tokens,
            "modalities": ["text", "audio"] if args.speech else ["text"], "temperature": 0.0}
    if args.audio:
        with open(args.audio, "rb") as f:
            body["audios"] = ["data:audio/wav;base64," + base64.b64encode(f.read()).decode()]
    pcm, rate = [], 24000
    with httpx.stream("POST", f"{args.url}/v1/chat/completions", json=body, timeout=600) as r:
        for line in r.iter_lines():
            if not line.startswith("data:") or line.strip() == "data: [DONE]":
                continue
            msg = json.loads(line[5:])
            delta = (msg.get("choices") or [{}])[0].get("delta") or {}
            if delta.get("content"):
                print(delta["content"], end="", flush=True)
            if (delta.get("audio") or {}).get("data"):
                p, rate = _pcm_of(base64.b64decode(delta["audio"]["data"]))
                pcm.append(p)
    print()
    if pcm:
        with wave.open(args.out, "wb") as w:
            w.setnchannels(1)
            w.setsampwidth(2)
            w.setframerate(rate)
            w.writeframes(b"".join(pcm))
        print(f"speech written to {args.out}")
    if args.tts:
        r = httpx.post(f"{args.url}/v1/audio/speech", json={"input": args.tts, "response_format": "wav"}, timeout=600)
        r.raise_for_status()
        with open("tts.wav", "wb") as f:
            f.write(r.content)
        print("tts.wav written")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--url", default="http://localhost:8000")
    ap.add_argument("--prompt", default="Hello! Who are you?")
    ap.add_argument("--audio", help="WAV file sent as input audio")
    ap.add_argument("--speech", action="store_true", help="ask for speech output too")
    ap.add_argument("--max-tokens", type=int, default=128)
    ap.add_argument("--out", default="reply.wav")
    ap.add_argument("--tts", help="also synthesise this text through /v1/audio/speech (S2-Pro servers)")
    main(ap.parse_args())
