"""B200-native (sm_100a) JoLT / FlashJoLT KV-cache compression."""
