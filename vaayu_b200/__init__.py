"""vaayu_b200: B200-native fused packed-int4 MoE expert path."""
