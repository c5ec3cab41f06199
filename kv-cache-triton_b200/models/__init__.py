"""Drop-in replacements for the reference's ``models`` package (INT4 KV-cache
glue for Llama 3.1 and GPT-2), backed by libkvint4.so."""
