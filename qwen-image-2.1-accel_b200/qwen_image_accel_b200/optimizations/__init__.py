"""Pipeline-scoped optimization policies (mirrors qwen_image_accel.optimizations)."""
