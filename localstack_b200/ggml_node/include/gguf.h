// gguf.h - the one GGUF name the reference's model headers mention: the parsed file, defined by
// the front end's own GGUF reader (node.cu).
#pragma once

struct gguf_context;
