"""GLM-4.7-Flash plugin (counterpart of ``pio/models/glm_4_7_flash/plugin.py``)."""
from typing import Dict, List, Optional

from ....api.engine_plugin import EnginePlugin


class GLM_4_7_Flash_Plugin(EnginePlugin):
    preset = "glm-4.7-flash"
    display_name = "GLM-4.7-Flash"
    family = "GLM"
    architecture = "GLM transformer (GQA, qkv bias, GELU MLP)"
    size = "flash"
    modalities = ('text',)

    def format_chat(self, messages: List[Dict[str, str]], enable_thinking: Optional[bool] = None) -> str:
        """GLM chat layout: ``[gMASK]<sop>`` then ``<|role|>`` headers, the reply after ``<|assistant|>``
        (with ``/nothink`` appended to the last user turn when thinking is off)."""
        think = self.thinking_default if enable_thinking is None else enable_thinking
        out = "[gMASK]<sop>"
        for i, m in enumerate(messages):
            body = m.get("content", "")
            if not think and m.get("role", "user") == "user" and i == len(messages) - 1:
                body += "/nothink"
            out += f"<|{m.get('role', 'user')}|>\n{body}"
        return out + "<|assistant|>\n"


def create_glm_4_7_flash_plugin():
    return GLM_4_7_Flash_Plugin()
