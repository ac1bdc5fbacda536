from .process import main

raise SystemExit(main())
