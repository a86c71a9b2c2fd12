"""Multi-turn chat sessions: templates, context trimming, streaming, think / critique modes.

Reference: ``mamformer/chat.py`` (``Message`` 64-72, ``ChatTemplate`` 75-120 with the built-in
Llama-2, Llama-3, simple, think and self-critique templates 122-178, ``ChatSession`` 183-682,
``create_chat`` 685-716).  The template strings are kept verbatim (they define the prompt
format a model was trained on), as are the session's JSON layout (``to_dict``) and its default
sampling settings.  Prompts are token-counted once per message; the oldest non-system messages
are dropped first when the history no longer leaves room for ``max_new_tokens``.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from typing import Generator, List, Optional, Tuple

import torch


@dataclass
class Message:
    role: str
    content: str
    token_count: int = 0


class ChatTemplate:
    def __init__(self, bos_token: str = "<s>", eos_token: str = "</s>", system_start: str = "<s>[INST] <<SYS>>\n",
                 system_end: str = "\n<</SYS>>\n\n", user_start: str = "<s>[INST] ", user_end: str = " [/INST]",
                 assistant_start: str = " ", assistant_end: str = " </s>"):
        self.bos_token, self.eos_token = bos_token, eos_token
        self.system_start, self.system_end = system_start, system_end
        self.user_start, self.user_end = user_start, user_end
        self.assistant_start, self.assistant_end = assistant_start, assistant_end

    def format_message(self, message: Message) -> str:
        wrap = {"system": (self.system_start, self.system_end), "user": (self.user_start, self.user_end),
                "assistant": (self.assistant_start, self.assistant_end)}.get(message.role)
        return message.content if wrap is None else wrap[0] + message.content + wrap[1]

    def format_conversation(self, messages: List[Message]) -> str:
        return "".join(self.format_message(m) for m in messages)


LLAMA2_CHAT_TEMPLATE = ChatTemplate()
LLAMA3_CHAT_TEMPLATE = ChatTemplate(
    bos_token="<|begin_of_text|>", eos_token="<|eos_token|>",
    system_start="<|start_header_id|>system<|end_header_id|>\n\n", system_end="<|eot_id|>",
    user_start="<|start_header_id|>user<|end_header_id|>\n\n", user_end="<|eot_id|>",
    assistant_start="<|start_header_id|>assistant<|end_header_id|>\n\n", assistant_end="<|eot_id|>")
SIMPLE_CHAT_TEMPLATE = ChatTemplate(bos_token="", eos_token="", system_start="System: ", system_end="\n",
                                    user_start="User: ", user_end="\n", assistant_start="Assistant: ",
                                    assistant_end="\n")
REFLECTION_SYSTEM_PROMPT = ("Before answering, think carefully about the question. "
                            "Consider multiple perspectives, check for errors in your reasoning, "
                            "and only then provide your final answer.")
THINK_TEMPLATE = ChatTemplate(assistant_start="<thinking>\n", assistant_end="\n</thinking>\n\n<answer>\n")
SELF_CRITIQUE_TEMPLATE = ChatTemplate(
    assistant_start="<draft>\n",
    assistant_end=("\n</draft>\n\n<critique>\nReview the above draft for errors, bias, or missing information. "
                   "Then provide the improved answer:\n</critique>\n\n<final>\n"))

_STOP_MARKERS = ("\nUser:", "\nSystem:", "\n<s>", "\n[INST]", "\n<|start_header_id|>", "\nHuman:",
                 "\nAssistant:", "\n\nUser", "User: ")
_TEMPLATE_MARKERS = ("<s>[INST] ", " [/INST]", "</s>", "<|eot_id|>", "Assistant: ", "<answer>", "<thinking>",
                     "</thinking>", "<final>", "</final>", "<draft>", "</draft>", "<critique>", "</critique>")


class ChatSession:
    def __init__(self, model, tokenizer, system_prompt: Optional[str] = None, max_context: int = 4096,
                 template: Optional[ChatTemplate] = None, device: str = "cpu", reflection_mode: str = "none"):
        self.model, self.tokenizer = model, tokenizer
        self.max_context = max_context
        self.template = template or ChatTemplate()
        self.device = device
        self.reflection_mode = reflection_mode
        self.messages: List[Message] = []
        self.temperature, self.top_k, self.top_p = 0.7, 50, 0.9
        self.max_new_tokens = 512
        self.repetition_penalty = 1.0
        self.think_tokens, self.critique_tokens = 256, 128
        self.show_thinking = False
        self._last_thinking = ""
        if system_prompt:
            self.set_system_prompt(system_prompt)

    # -- history -------------------------------------------------------------------------------
    def _count_tokens(self, text: str) -> int:
        return len(self.tokenizer.encode(text, add_bos=False, add_eos=False))

    def set_system_prompt(self, prompt: str) -> None:
        msg = Message("system", prompt, self._count_tokens(prompt))
        if self.messages and self.messages[0].role == "system":
            self.messages[0] = msg
        else:
            self.messages.insert(0, msg)

    def get_system_prompt(self) -> Optional[str]:
        return self.messages[0].content if self.messages and self.messages[0].role == "system" else None

    def add_user_message(self, content: str) -> None:
        self.messages.append(Message("user", content, self._count_tokens(content)))

    def add_assistant_message(self, content: str) -> None:
        self.messages.append(Message("assistant", content, self._count_tokens(content)))

    def get_history(self) -> List[dict]:
        return [{"role": m.role, "content": m.content} for m in self.messages]

    def get_formatted_prompt(self) -> str:
        return self.template.format_conversation(self.messages)

    def clear_history(self, keep_system: bool = True) -> None:
        sys_msg = self.messages[:1] if (keep_system and self.messages and self.messages[0].role == "system") else []
        self.messages = sys_msg

    def get_token_count(self) -> int:
        return sum(m.token_count for m in self.messages)

    def _trim_to_context(self) -> None:
        budget = self.max_context - self.max_new_tokens
        while self.get_token_count() > budget:
            idx = next((i for i, m in enumerate(self.messages) if m.role != "system"), None)
            if idx is None:
                break
            self.messages.pop(idx)

    # -- prompting -------------------------------------------------------------------------------
    def _prompt_ids(self, template: ChatTemplate, strip_markers: bool = False) -> List[int]:
        self._trim_to_context()
        prompt = template.format_conversation(self.messages)
        if strip_markers:
            prompt = self._clean_prompt_for_template(prompt, template)
        else:
            if self.messages and self.messages[-1].role == "assistant" and template.assistant_end \
                    and prompt.endswith(template.assistant_end):
                prompt = prompt[:-len(template.assistant_end)]
            prompt += template.assistant_start
        ids = self.tokenizer.encode(prompt, add_bos=False)
        if len(ids) > self.max_context:
            raise RuntimeError(f"Prompt length ({len(ids)}) exceeds max_context ({self.max_context}). "
                               "Reduce conversation length or increase max_context.")
        return ids

    def _generate_text(self, ids: List[int], max_new: int, eos: Optional[int]) -> str:
        x = torch.tensor([ids], device=self.device)
        out = self.model.generate(input_ids=x, max_new_tokens=max_new, temperature=self.temperature,
                                  top_k=self.top_k, top_p=self.top_p, eos_token_id=eos,
                                  pad_token_id=getattr(self.tokenizer, "pad_token_id", None))
        full = self.tokenizer.decode(out[0].tolist(), skip_special_tokens=True)
        head = self.tokenizer.decode(ids, skip_special_tokens=True)
        return full[len(head):] if full.startswith(head) else full

    @torch.no_grad()
    def generate_response(self) -> str:
        ids = self._prompt_ids(self.template)
        resp = self._clean_response(self._generate_text(ids, self.max_new_tokens, self.tokenizer.eos_token_id).strip())
        self.add_assistant_message(resp)
        return resp

    @torch.no_grad()
    def generate_stream(self) -> Generator[str, None, None]:
        from mamformer_b200.sampling import sample_one_token
        ids = self._prompt_ids(self.template)
        seq = torch.tensor([ids], device=self.device)
        cache, text = None, ""
        for _ in range(self.max_new_tokens):
            out = self.model(input_ids=seq[:, -1:] if cache is not None else seq, use_cache=True, cache=cache,
                             rope_offset=0)
            cache = out.get("cache")
            nxt = sample_one_token(out["logits"][:, -1, :], temperature=self.temperature, top_k=self.top_k,
                                   top_p=self.top_p)
            seq = torch.cat([seq, nxt], -1)
            tid = int(nxt[0, 0])
            piece = self.tokenizer.decode([tid], skip_special_tokens=True)
            text += piece
            yield piece
            if tid == self.tokenizer.eos_token_id:
                break
        resp = self._clean_response(text)
        if resp:
            self.add_assistant_message(resp)

    @torch.no_grad()
    def generate_with_reflection(self) -> str:
        if self.reflection_mode == "think":
            return self._generate_with_thinking()
        if self.reflection_mode == "critique":
            return self._generate_with_critique()
        return self.generate_response()

    def _generate_with_thinking(self) -> str:
        ids = self._prompt_ids(THINK_TEMPLATE, strip_markers=True)
        resp = self._generate_text(ids, self.think_tokens + self.max_new_tokens, None)   # no early EOS
        thinking, answer = self._parse_thinking_response(resp)
        self._last_thinking = thinking
        hist = f"[thinking]\n{thinking}\n[/thinking]\n\n{answer}" if self.show_thinking else answer
        self.add_assistant_message(self._clean_response(hist))
        return answer

    def _generate_with_critique(self) -> str:
        ids = self._prompt_ids(SELF_CRITIQUE_TEMPLATE, strip_markers=True)
        resp = self._generate_text(ids, 2 * self.max_new_tokens + self.critique_tokens, self.tokenizer.eos_token_id)
        final = self._parse_critique_response(resp) or resp
        self._last_thinking = resp
        self.add_assistant_message(self._clean_response(final))
        return final

    # -- parsing -------------------------------------------------------------------------------
    @staticmethod
    def _parse_thinking_response(text: str) -> Tuple[str, str]:
        if "<thinking>" in text and "</thinking>" in text:
            a = text.find("<thinking>") + len("<thinking>")
            b = text.find("</thinking>")
            rest = text[b + len("</thinking>"):]
            ans = rest[rest.find("<answer>") + len("<answer>"):] if "<answer>" in rest else rest
            return text[a:b].strip(), ans.strip()
        return "", text

    @staticmethod
    def _parse_critique_response(text: str) -> str:
        if "<final>" in text:
            t = text[text.rfind("<final>") + len("<final>"):].strip()
            return t[:t.find("</final>")].strip() if "</final>" in t else t
        if "</critique>" in text:
            return text[text.rfind("</critique>") + len("</critique>"):].strip()
        return text.strip()

    @staticmethod
    def _clean_prompt_for_template(prompt: str, template: ChatTemplate) -> str:
        out = prompt
        for mk in _TEMPLATE_MARKERS:
            if out.strip().endswith(mk.strip()):
                out = out[:out.rfind(mk)]
        return out.strip()

    def get_last_thinking(self) -> str:
        return self._last_thinking

    @staticmethod
    def _clean_response(text: str) -> str:
        for mk in _STOP_MARKERS:
            i = text.find(mk)
            if i > 0:
                text = text[:i]
        return text.strip()

    # -- persistence -------------------------------------------------------------------------------
    def to_dict(self) -> dict:
        return {"messages": self.get_history(), "system_prompt": self.get_system_prompt(),
                "config": {"max_context": self.max_context, "temperature": self.temperature, "top_k": self.top_k,
                           "top_p": self.top_p, "max_new_tokens": self.max_new_tokens,
                           "repetition_penalty": self.repetition_penalty, "reflection_mode": self.reflection_mode}}

    @classmethod
    def from_dict(cls, data: dict, model, tokenizer, device: str = "cpu") -> "ChatSession":
        c = data.get("config", {})
        s = cls(model, tokenizer, system_prompt=data.get("system_prompt"), max_context=c.get("max_context", 4096),
                device=device, reflection_mode=c.get("reflection_mode", "none"))
        s.temperature = c.get("temperature", 0.7)
        s.top_k = c.get("top_k", 50)
        s.top_p = c.get("top_p", 0.9)
        s.max_new_tokens = c.get("max_new_tokens", 512)
        s.repetition_penalty = c.get("repetition_penalty", 1.0)
        for m in data.get("messages", []):
            if m["role"] == "user":
                s.add_user_message(m["content"])
            elif m["role"] == "assistant":
                s.add_assistant_message(m["content"])
        return s

    def save(self, path: str) -> None:
        with open(path, "w", encoding="utf-8") as f:
            json.dump(self.to_dict(), f, ensure_ascii=False, indent=2)

    @classmethod
    def load(cls, path: str, model, tokenizer, device: str = "cpu") -> "ChatSession":
        with open(path, "r", encoding="utf-8") as f:
            return cls.from_dict(json.load(f), model, tokenizer, device)


def create_chat(model, tokenizer, system_prompt: Optional[str] = None, max_context: Optional[int] = None,
                device: str = "cpu") -> ChatSession:
    if max_context is None and hasattr(model, "config"):
        max_context = model.config.generation.max_context
    return ChatSession(model, tokenizer, system_prompt=system_prompt, max_context=max_context or 4096, device=device)
