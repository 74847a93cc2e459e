// gguf.h - the one GGUF name the reference's model headers mention (an opaque parsed file). The
// front end builds its weights directly and never parses GGUF.
#pragma once

struct gguf_context;
