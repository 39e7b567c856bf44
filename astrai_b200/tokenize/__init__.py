from astrai_b200.tokenize.tokenizer import AutoTokenizer, ChatTemplate, Message, Messages

__all__ = ["AutoTokenizer", "ChatTemplate", "Message", "Messages"]
