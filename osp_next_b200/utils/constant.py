"""Dictionary keys and the default negative prompt.

The keys and the default (Chinese, Wan-2.1) negative prompt are data constants that
must equal the reference's (ospnext/utils/constant.py) so that cached text
embeddings and datasets interoperate.
"""
VIDEO = "video"
IMAGE = "image"
VIDEO_MASK = "video_mask"
PROMPT = "prompt"
PROMPT_IDS = "prompt_ids"
PROMPT_MASK = "prompt_mask"
START_FRAME = "start_frame"
NAME_INDEX = "name_index"
NEGATIVE_PROMPT = "色调艳丽，过曝，静态，细节模糊不清，字幕，风格，作品，画作，画面，静止，整体发灰，最差质量，低质量，JPEG压缩残留，丑陋的，残缺的，多余的手指，画得不好的手部，画得不好的脸部，畸形的，毁容的，形态畸形的肢体，手指融合，静止不动的画面，杂乱的背景，三条腿，背景人很多，倒着走"
