"""B200-native Whisper text-decoder token loop (drop-in for whisper4j's WhisperDecoder path)."""
